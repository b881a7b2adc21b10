"""ReaxFF (LAMMPS conventions): every energy term, the equilibrated charges and forces against
golden values computed with the reference package's own ReaxFF on CPU (a CHO molecule pair, a
periodic 96-atom water box, and a CHNO set with a C-O triple bond and acetylene under another
library); finite differences; permutation and rotation invariance."""
import json
from pathlib import Path

import pytest
import torch

from xnn_b200.data import structure_to_graph, synthetic
from xnn_b200.ffnn.reaxff import ReaxFF, ReaxFFLibrary

GOLD = json.loads((Path(__file__).parent / "data" / "reaxff_gold.json").read_text())


@pytest.fixture(autouse=True)
def _f64():
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(prev)


def _case(name):
    rec = GOLD[name]
    if name == "waterbox":
        s = synthetic.water_box(96, seed=5)
        s = {"pos": s["pos"].double(), "atomic_numbers": s["atomic_numbers"], "cell": s["cell"].double(),
             "pbc": torch.ones(3, dtype=torch.bool)}
    else:
        s = {"pos": torch.tensor(rec["pos"]), "atomic_numbers": torch.tensor(rec["z"])}
    return rec, s


def test_library_reading():
    lib = ReaxFFLibrary("CHO_cho_2008")
    assert lib.species == ["H", "C", "O"]
    assert lib.general["p_boc1"] == 50.0 and lib.general["swb"] == 10.0
    assert lib.atoms["O"]["valency_val"] == 4.0 and lib.bonds[("C", "C")]["De_p"] == 100.04
    assert lib.hbonds[("O", "H", "O")]["r0_hb"] == 1.9682
    assert lib.torsion("H", "C", "C", "H")["V2"] == 30.0252 and lib.torsion("O", "C", "H", "H")["V2"] == 0.0
    assert lib.torsion("H", "O", "C", "N") is None


@pytest.mark.parametrize("name", ["cho", "waterbox", "chno"])
def test_terms_charges_forces_match_reference(name):
    rec, s = _case(name)
    m = ReaxFF(rec["lib"])
    g = structure_to_graph(s, m.cutoff)
    g.pos.requires_grad_(True)
    out = m(g)
    for k, v in rec.items():
        if k.startswith("e_") or k == "energy":
            assert float(out[k].detach().sum()) == pytest.approx(v, abs=5e-7, rel=1e-8), k
    assert torch.allclose(out["charges"][:3], torch.tensor(rec["charges3"]), atol=1e-8)
    f = -torch.autograd.grad(out["energy"].sum(), g.pos)[0]
    assert torch.allclose(f[0], torch.tensor(rec["f0"]), atol=5e-5)
    assert torch.allclose(f[5], torch.tensor(rec["f5"]), atol=5e-5)


def test_finite_difference_and_invariance():
    rec, s = _case("cho")
    m = ReaxFF("CHO_cho_2008")
    g = structure_to_graph(s, m.cutoff)
    g.pos.requires_grad_(True)
    out = m(g)
    e = out["energy"].sum()
    f = -torch.autograd.grad(e, g.pos)[0]
    # the forces hold the equilibrated charges fixed: so does the finite difference
    q0 = out["charges"].detach()
    m._qeq = lambda *a, **k: q0
    h = 1e-6
    for a, c in [(0, 0), (3, 2), (9, 1)]:
        sp = dict(s, pos=s["pos"].clone())
        sm = dict(s, pos=s["pos"].clone())
        sp["pos"][a, c] += h
        sm["pos"][a, c] -= h
        fd = -(float(m(structure_to_graph(sp, m.cutoff))["energy"]) - float(m(structure_to_graph(sm, m.cutoff))["energy"]))
        assert fd / (2 * h) == pytest.approx(float(f[a, c]), abs=2e-4)
    gen = torch.Generator().manual_seed(0)
    rot, _ = torch.linalg.qr(torch.randn(3, 3, generator=gen))
    perm = torch.randperm(s["pos"].shape[0], generator=gen)
    s2 = {"pos": s["pos"][perm] @ rot.T, "atomic_numbers": s["atomic_numbers"][perm]}
    del m._qeq
    e2 = m(structure_to_graph(s2, m.cutoff))["energy"]
    assert float(e2) == pytest.approx(float(e), abs=1e-9)


@pytest.mark.gpu
def test_cuda_matches_cpu():
    rec, s = _case("waterbox")
    m = ReaxFF(rec["lib"])
    g = structure_to_graph(s, m.cutoff)
    out_c = m(g)
    gg = g.to("cuda")
    gg.pos.requires_grad_(True)
    out_g = m.to("cuda")(gg)
    for k in ("energy", "e_bond", "e_angle", "e_hbond", "e_coulomb"):
        assert float(out_g[k].sum()) == pytest.approx(float(out_c[k].sum()), abs=1e-8), k
    f = -torch.autograd.grad(out_g["energy"].sum(), gg.pos)[0]
    assert torch.isfinite(f).all()
