"""AMOEBA: the parameter reader, local frames, every energy term against golden values computed
with the reference package's own AMOEBA on CPU (a perturbed water dimer, and a periodic 648-atom
water box on a 64^3 mesh), finite-difference forces, invariances and the GPU path."""
import math

import pytest
import torch

from xnn_b200.data import structure_to_graph, synthetic
from xnn_b200.ffnn.amoeba import Amoeba, ewald_coefficient
from xnn_b200.ffnn.amoeba_params import amoeba_water_2003, parse_prm
from xnn_b200.ffnn.multipoles import DEBYE, EwaldSetup

# perturbed Smith dimer 1 (Angstrom)
DIMER = [[0.8740975110546697, -0.006605243164565094, -1.171628867477836],
         [0.329890005857652, -0.02678346865805555, -1.9720022472545258],
         [0.30536900225650687, 0.04735404815646211, -0.5065427617903496],
         [-0.8877820735523027, -0.03116372312686761, 1.1472922989673622],
         [-0.7422605387319418, 0.7481454168033728, 1.6320414526373468],
         [-0.6626223677351726, -0.7862979491428655, 1.6785219921815422]]
# the reference package's AMOEBA (amoeba-water-2003) on DIMER, eV and eV/A
GOLD_DIMER = {"energy": 0.03398888285258425, "e_bond": 0.20577922898319476, "e_angle": 0.0055044420570438055,
              "e_urey": 0.012764649055384625, "e_vdw": 0.06385263082029843, "e_multipole": -0.21383737937369268,
              "e_polar": -0.04007468868964469}
GOLD_F0 = [2.9010166237335495, -0.28230578133031603, -4.387392721566279]
GOLD_F4 = [0.25190673531849384, 1.2580319892394058, 0.8866705272861857]
# the same on synthetic.water_box(648, seed=3), cutoff 9 A, Ewald real-space cutoff 7 A, 64^3 mesh
GOLD_BOX = {"energy": -4.183698462712765, "e_vdw": 2.9554470936578365, "e_multipole": 1.1988077151387246,
            "e_polar": -10.511600321979907, "e_bond": 0.07722878243639013, "e_angle": 1.642967384149725,
            "e_urey": 0.45345088388446697}
GOLD_BOX_F = {0: [0.16261497359454144, -0.36795064021452734, 0.3067653528383894],
              100: [0.06365195523385261, -0.04738222947822438, 0.45770379110294845],
              401: [-0.5574473272546254, 0.0395499418728907, -0.021575232599262945]}


@pytest.fixture(autouse=True)
def _f64():
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(prev)


def _graph(pos, z, cutoff=30.0, cell=None):
    s = {"pos": torch.as_tensor(pos, dtype=torch.float64), "atomic_numbers": torch.as_tensor(z)}
    if cell is not None:
        s["cell"] = torch.as_tensor(cell, dtype=torch.float64)
        s["pbc"] = torch.ones(3, dtype=torch.bool)
    return structure_to_graph(s, cutoff)


def _monomer(r=0.9572, theta=108.5):
    h = math.radians(theta) / 2
    return [[0.0, 0.0, 0.0], [r * math.sin(h), 0.0, r * math.cos(h)], [-r * math.sin(h), 0.0, r * math.cos(h)]]


def test_parameters_and_frames():
    p = amoeba_water_2003()
    assert p.types[1][:3] == (1, "O", 8) and p.vdw[2] == (2.655, 0.0135, 0.91)
    assert p.multipoles[1][0].frame == "bisector" and p.multipoles[2][0].frame == "z-then-x"
    assert p.polarize[1] == (0.837, 0.39, (2,))
    assert p.scale("mpole", 4) == 0.4 and p.group_scale("direct", 1) == 0.0 and p.group_scale("mutual", 1) == 1.0
    text = "atom 3 4 C \"x\" 6 12.0 4\nmultipole 3 4 -5 -6 0.1\n 0 0 0\n 0\n 0 0\n 0 0 0\n"
    q = parse_prm(text)
    assert q.types[3] == (4, "C", 6, 12.0) and q.multipoles[3][0].frame == "z-bisect"


def test_monomer_dipole_of_ren_and_ponder():
    """1.773 D at the 108.5 degree geometry (Table 2), along the bisector."""
    m = Amoeba.water(1)
    pos = torch.tensor(_monomer())
    q, d, Q = m.moments(pos)
    mu = (d.sum(0) + (q[:, None] * pos).sum(0)) / DEBYE
    assert float(mu.norm()) == pytest.approx(1.773, abs=2e-3)
    assert abs(float(mu[0])) < 1e-12 and float(mu[2]) > 0
    assert torch.allclose(Q.diagonal(dim1=1, dim2=2).sum(-1), torch.zeros(3), atol=1e-12)
    out = m(_graph(_monomer(), [8, 1, 1]))
    assert float(out["e_polar"]) == 0.0                    # one group: no induction within it


def test_dimer_matches_reference_terms_and_forces():
    m = Amoeba.water(2)
    g = _graph(DIMER, [8, 1, 1, 8, 1, 1])
    g.pos.requires_grad_(True)
    out = m(g)
    for k, v in GOLD_DIMER.items():
        assert float(out[k].sum()) == pytest.approx(v, abs=2e-9), k
    f = -torch.autograd.grad(out["energy"].sum(), g.pos)[0]
    assert torch.allclose(f[0], torch.tensor(GOLD_F0), atol=5e-9)
    assert torch.allclose(f[4], torch.tensor(GOLD_F4), atol=5e-9)


def test_forces_finite_difference_and_invariance():
    m = Amoeba.water(3)
    g = torch.Generator().manual_seed(1)
    pos = torch.tensor(DIMER + [[2.5, 2.4, 0.3], [3.2, 2.0, 0.8], [2.0, 3.0, 0.9]])
    pos = pos + 0.03 * torch.randn(pos.shape, generator=g)
    z = [8, 1, 1] * 3
    gr = _graph(pos, z)
    gr.pos.requires_grad_(True)
    e = m(gr)["energy"].sum()
    f = -torch.autograd.grad(e, gr.pos)[0]
    h = 1e-5
    for a, c in [(0, 0), (4, 1), (7, 2)]:
        pp, pm = pos.clone(), pos.clone()
        pp[a, c] += h
        pm[a, c] -= h
        fd = -(float(m(_graph(pp, z))["energy"]) - float(m(_graph(pm, z))["energy"])) / (2 * h)
        assert fd == pytest.approx(float(f[a, c]), abs=2e-6)
    rot, _ = torch.linalg.qr(torch.randn(3, 3, generator=g))
    rot = rot * torch.sign(torch.det(rot))
    g2 = _graph(pos @ rot.T + torch.tensor([1.0, -2.0, 0.5]), z)
    g2.pos.requires_grad_(True)
    e2 = m(g2)["energy"].sum()
    f2 = -torch.autograd.grad(e2, g2.pos)[0]
    assert float(e2) == pytest.approx(float(e), abs=1e-10)
    assert torch.allclose(f2, f @ rot.T, atol=1e-9)


def _box(device="cpu"):
    s = synthetic.water_box(648, seed=3)
    n = s["pos"].shape[0]
    m = Amoeba.water(n // 3, cutoff=9.0, ewald=EwaldSetup(alpha=ewald_coefficient(7.0), cutoff=7.0, mesh=(64, 64, 64),
                                                           order=5, fft_dtype=torch.float64)).to(device)
    g = _graph(s["pos"], s["atomic_numbers"], 9.0, s["cell"]).to(device)
    return m, g


def test_periodic_water_box_matches_reference():
    m, g = _box()
    g.pos.requires_grad_(True)
    out = m(g)
    for k, v in GOLD_BOX.items():
        tol = 1e-8 if k in ("e_vdw", "e_bond", "e_angle", "e_urey") else 3e-4
        assert float(out[k].sum()) == pytest.approx(v, abs=tol), k
    f = -torch.autograd.grad(out["energy"].sum(), g.pos)[0]
    for a, v in GOLD_BOX_F.items():
        assert torch.allclose(f[a], torch.tensor(v), atol=1e-5), a


@pytest.mark.gpu
def test_periodic_box_on_gpu_matches_cpu():
    m, g = _box()
    out_c = m(g)
    m2, g2 = _box("cuda")
    g2.pos.requires_grad_(True)
    out_g = m2(g2)
    for k in ("energy", "e_multipole", "e_polar", "e_vdw"):
        assert float(out_g[k].sum()) == pytest.approx(float(out_c[k].sum()), abs=1e-7), k
    f = -torch.autograd.grad(out_g["energy"].sum(), g2.pos)[0]
    assert torch.isfinite(f).all()


def test_tinker_inputs_round_trip(tmp_path):
    from xnn_b200.ffnn.amoeba_params import read_tinker_xyz, parse_prm
    m = Amoeba.water(2)
    xyz, key, prm = m.write_tinker_inputs(tmp_path, DIMER, cell=[[12.0, 0, 0], [0, 12.0, 0], [0, 0, 12.0]])
    pos, types, bonds, syms, cell = read_tinker_xyz(xyz)
    assert types == [1, 2, 2, 1, 2, 2] and syms == ["O", "H", "H", "O", "H", "H"]
    assert bonds == [(0, 1), (0, 2), (3, 4), (3, 5)]
    assert abs(pos - torch.tensor(DIMER).numpy()).max() < 1e-6 and abs(cell - 12.0 * torch.eye(3).numpy()).max() < 1e-6
    assert "parameters  system.prm" in key.read_text() and "ewald" in key.read_text()
    assert parse_prm(prm.read_text()).bonds == m.params.bonds
