"""D3 dispersion and LES Ewald sums against the reference framework's own CPU implementations
(used as oracles when installed under baseline/_ref), plus wrapper plumbing."""
import os
import sys

import pytest
import torch

from xnn_b200.data import structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _reference(module):
    if not os.path.isdir(os.path.join(REF, "xnn")):
        pytest.skip("reference framework not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import importlib
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        return importlib.import_module(module)


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _d3_inputs(kind):
    if kind == "molecule":
        s = synthetic.organic_molecules(1, seed=4, labels=False)[0]
        cut = 20.0
    else:
        s = synthetic.triclinic_crystals(1, seed=2, labels=False)[0]
        s["pos"], s["atomic_numbers"] = s["pos"][:12], s["atomic_numbers"][:12]
        cut = 12.0
    return s, cut


@pytest.mark.parametrize("kind", ["molecule", "crystal"])
@pytest.mark.parametrize("damping,s9", [("bj", 0.0), ("zero", 0.0), ("bj", 1.0), ("mzero", 0.0), ("op", 0.0)])
def test_d3_matches_reference(kind, damping, s9):
    ref_d3 = _reference("xnn.common.models.d3")
    from xnn_b200.models.d3 import DFTD3
    s, cut = _d3_inputs(kind)
    opts = dict(damping=damping, s9=s9, cutoff_pair=cut, cutoff_triple=cut * 0.8, cutoff_cn=cut * 0.8,
                bet=0.3 if damping in ("mzero", "op") else 0.0)
    mine, theirs = DFTD3(**opts), ref_d3.DFTD3(**opts)
    g = structure_to_graph(s, cut)
    pos = g.pos.clone().requires_grad_(True)
    args = lambda p: (g.atomic_numbers, p, g.edge_index,  # noqa: E731
                      p[g.edge_index[1]] - p[g.edge_index[0]] + (g.cell_shifts.double() @ g.cell[0]
                                                                 if g.cell is not None else 0.0),
                      g.batch, 1, torch.zeros(1, 3, 3), torch.zeros(1, 3, dtype=torch.bool), torch.zeros(1))
    a = mine.evaluate(*args(pos))
    b = theirs.evaluate(*args(pos))
    torch.testing.assert_close(a["node_energy"], b["node_energy"], rtol=1e-9, atol=1e-11)
    torch.testing.assert_close(a["coordination_numbers"], b["coordination_numbers"], rtol=1e-11, atol=1e-12)
    fa, = torch.autograd.grad(a["node_energy"].sum(), pos, retain_graph=True)
    fb, = torch.autograd.grad(b["node_energy"].sum(), pos)
    torch.testing.assert_close(fa, fb, rtol=1e-8, atol=1e-11)


def test_d3_wrapper_adds_to_model():
    from xnn_b200.models.d3 import D3Dispersion
    from xnn_b200.models.mace import MACE
    torch.manual_seed(0)
    m = MACE(species=[1, 6, 7, 8, 9, 16, 17], cutoff=4.5, num_channels=8, n_rbf=6, num_interactions=1,
             max_ell=1, correlation=2, avg_num_neighbors=5.0)
    w = D3Dispersion(model=m, cutoff_pair=10.0, cutoff_cn=8.0, cutoff_triple=8.0)
    assert w.cutoff == 10.0
    s = synthetic.organic_molecules(1, seed=4, labels=False)[0]
    g = structure_to_graph(s, w.cutoff)
    out = ForceStressOutput(w)(g)
    sr = ForceStressOutput(m)(structure_to_graph(s, 4.5))
    d3 = ForceStressOutput(D3Dispersion(cutoff_pair=10.0, cutoff_cn=8.0, cutoff_triple=8.0))(g)
    torch.testing.assert_close(out["energy"], sr["energy"] + d3["energy"], rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(out["forces"], sr["forces"] + d3["forces"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("exponent", [1, 6])
def test_ewald_reciprocal_matches_reference(exponent):
    les_ref = _reference("xnn.common.models.les")
    from xnn_b200.models.les import EwaldSummation
    g = torch.Generator().manual_seed(3)
    cell = torch.tensor([[9.0, 0.3, 0.0], [0.5, 8.0, 0.2], [0.1, -0.4, 10.0]])
    pos = (torch.rand(40, 3, generator=g) @ cell).requires_grad_(True)
    q = torch.randn(40, 3, generator=g)
    mine = EwaldSummation(dl=1.5, sigma=1.0, exponent=exponent, atom_block=7)
    theirs = les_ref.EwaldSummation(dl=1.5, sigma=1.0, exponent=exponent)
    a = mine.reciprocal(pos, q, cell)
    b = theirs.reciprocal(pos, q, cell)
    torch.testing.assert_close(a, b, rtol=1e-12, atol=1e-12)
    ga, = torch.autograd.grad(a, pos)
    gb, = torch.autograd.grad(b, pos)
    torch.testing.assert_close(ga, gb, rtol=1e-10, atol=1e-12)


def test_ewald_realspace_matches_reference():
    les_ref = _reference("xnn.common.models.les")
    from xnn_b200.models.les import EwaldSummation
    g = torch.Generator().manual_seed(5)
    pos = torch.randn(30, 3, generator=g) * 3
    q = torch.randn(30, 2, generator=g)
    batch = torch.repeat_interleave(torch.arange(3), torch.tensor([10, 12, 8]))
    mine, theirs = EwaldSummation(sigma=0.8), les_ref.EwaldSummation(sigma=0.8)
    torch.testing.assert_close(mine.realspace_batch(pos, q, batch, 3), theirs.realspace_batch(pos, q, batch, 3),
                               rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(mine.realspace_single(pos, q), theirs.realspace_single(pos, q), rtol=1e-12,
                               atol=1e-12)


def test_latent_ewald_wrapper():
    from xnn_b200.models.les import LatentEwald
    from xnn_b200.models.mace import MACE
    torch.manual_seed(0)
    m = MACE(species=[1, 6, 7, 8, 9, 16, 17], cutoff=4.5, num_channels=8, n_rbf=6, num_interactions=2,
             max_ell=2, correlation=2, avg_num_neighbors=5.0)
    les = LatentEwald(m, n_channels=2, constrain_charge=True)
    from xnn_b200.data import collate
    mols = synthetic.organic_molecules(2, seed=1, labels=False)
    b = collate([structure_to_graph(s, 4.5) for s in mols])
    out = ForceStressOutput(les)(b)
    torch.testing.assert_close(out["energy"], out["energy_sr"] + out["energy_lr"])
    # the constraint makes every structure neutral in every channel
    from xnn_b200.ops.scatter import scatter_sum
    torch.testing.assert_close(scatter_sum(out["latent_charges"], b.batch, 2), torch.zeros(2, 2), atol=1e-10,
                               rtol=0)
    assert out["forces"].shape == b.pos.shape
    # periodic structure through the reciprocal sum, forces by finite differences
    s = synthetic.triclinic_crystals(1, seed=3, labels=False)[0]
    s["atomic_numbers"] = torch.full_like(s["atomic_numbers"], 6)
    g1 = structure_to_graph(s, 4.5)
    o = ForceStressOutput(les)(g1.clone())
    k = 3
    eps = 1e-5
    gp, gm = g1.clone(), g1.clone()
    gp.pos = gp.pos.clone(); gm.pos = gm.pos.clone()
    gp.pos[k, 0] += eps
    gm.pos[k, 0] -= eps
    fd = -(les(gp)["energy"] - les(gm)["energy"]) / (2 * eps)
    torch.testing.assert_close(o["forces"][k, 0], fd[0], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("s9", [0.0, 1.0])
def test_d4_matches_reference_for_molecules(s9):
    ref_d4 = _reference("xnn.common.models.d4")
    from xnn_b200.data import collate
    from xnn_b200.models.d4 import DFTD4
    mols = synthetic.organic_molecules(2, seed=6, labels=False)
    b = collate([structure_to_graph(s, 14.0) for s in mols])
    opts = dict(s9=s9, cutoff_pair=14.0, cutoff_triple=10.0, cutoff_cn=10.0, cutoff_eeq_cn=10.0)
    mine, theirs = DFTD4(**opts), ref_d4.DFTD4(regime="dense", **opts)
    pos = b.pos.clone().requires_grad_(True)
    vec = pos[b.edge_index[1]] - pos[b.edge_index[0]]
    args = (b.atomic_numbers, pos, b.edge_index, vec, b.batch, 2, torch.zeros(2, 3, 3),
            torch.zeros(2, 3, dtype=torch.bool), torch.tensor([0.0, 1.0]))
    a = mine.evaluate(*args)
    r = theirs.evaluate(*args)
    for k in ("charges", "coordination_numbers", "polarizabilities"):
        torch.testing.assert_close(a[k], r[k], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(a["node_energy"], r["node_energy"], rtol=1e-9, atol=1e-11)
    fa, = torch.autograd.grad(a["node_energy"].sum(), pos, retain_graph=True)
    fr, = torch.autograd.grad(r["node_energy"].sum(), pos)
    torch.testing.assert_close(fa, fr, rtol=1e-8, atol=1e-11)


@pytest.mark.parametrize("s9", [0.0, 1.0])
def test_d4_matches_reference_for_crystals(s9):
    ref_d4 = _reference("xnn.common.models.d4")
    from xnn_b200.data import collate
    from xnn_b200.models.d4 import DFTD4
    from xnn_b200.models.outputs import ForceStressOutput
    xs = synthetic.triclinic_crystals(2, seed=5, labels=False)
    for s, z in zip(xs, ([8, 1], [6, 7, 1])):
        s["atomic_numbers"] = torch.as_tensor(z)[torch.arange(len(s["atomic_numbers"])) % len(z)]
    cut = 7.0
    b = collate([structure_to_graph(s, cut) for s in xs])
    opts = dict(s9=s9, cutoff_pair=cut, cutoff_triple=5.0, cutoff_cn=cut, cutoff_eeq_cn=cut)
    mine, theirs = DFTD4(**opts), ref_d4.DFTD4(regime="dense", **opts)
    args = lambda pos: (b.atomic_numbers, pos, b.edge_index, pos[b.edge_index[1]] - pos[b.edge_index[0]]  # noqa: E731
                        + b.cell_shifts.to(pos.dtype).unsqueeze(-1).mul(b.cell[b.batch[b.edge_index[0]]]).sum(1),
                        b.batch, 2, b.cell, b.pbc, torch.tensor([0.0, 0.0]))
    pos = b.pos.clone().requires_grad_(True)
    a, r = mine.evaluate(*args(pos)), theirs.evaluate(*args(pos))
    torch.testing.assert_close(a["charges"], r["charges"], rtol=1e-9, atol=1e-11)
    torch.testing.assert_close(a["node_energy"], r["node_energy"], rtol=1e-9, atol=1e-11)
    fa, = torch.autograd.grad(a["node_energy"].sum(), pos, retain_graph=True)
    fr, = torch.autograd.grad(r["node_energy"].sum(), pos)
    torch.testing.assert_close(fa, fr, rtol=1e-8, atol=1e-10)


@pytest.mark.gpu
@pytest.mark.parametrize("width", [0.0, 2.0])
def test_d4_three_body_kernel_matches_formulas(width):
    """The ATM kernel (energies per atom, forces, C6-factor gradients) against the tensor formulas."""
    _reference("xnn.common.models.d4")                      # the D4 reference tables
    from xnn_b200.data import collate
    from xnn_b200.models.d4 import DFTD4
    xs = synthetic.triclinic_crystals(2, seed=5, labels=False)
    cut = 7.0
    b = collate([structure_to_graph(s, cut) for s in xs]).to("cuda")
    opts = dict(s9=1.0, cutoff_pair=cut, cutoff_triple=6.0, cutoff_cn=cut, cutoff_eeq_cn=cut,
                switch_width_triple=width)
    m = DFTD4(**opts).to("cuda")

    def run(kernels):
        m.use_kernels = kernels
        pos = b.pos.clone().requires_grad_(True)
        vec = pos[b.edge_index[1]] - pos[b.edge_index[0]] + b.cell_shifts.to(pos.dtype).unsqueeze(-1).mul(
            b.cell[b.batch[b.edge_index[0]]]).sum(1)
        out = m.evaluate(b.atomic_numbers, pos, b.edge_index, vec, b.batch, 2, b.cell, b.pbc,
                         torch.zeros(2, device="cuda"))
        f, = torch.autograd.grad(out["energy_3body"].sum(), pos)
        return out, f

    a, fa = run(True)
    r, fr = run(False)
    torch.testing.assert_close(a["energy_3body"], r["energy_3body"], rtol=1e-11, atol=1e-13)
    torch.testing.assert_close(a["node_energy"], r["node_energy"], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(fa, fr, rtol=1e-9, atol=1e-12)


@pytest.mark.gpu
def test_d4_matrix_free_eeq_matches_dense():
    """Matrix-free EEQ (all-pairs product kernel, implicit derivatives) against the dense solve."""
    _reference("xnn.common.models.d4")
    from xnn_b200.models.d4 import DFTD4
    m = DFTD4(s9=0.0).to("cuda")
    s = synthetic.organic_molecules(1, seed=9, labels=False)[0]
    z = s["atomic_numbers"].to("cuda")
    gen = torch.Generator().manual_seed(0)
    pos0 = (s["pos"].double() / 0.529177210903).to("cuda")
    cn = torch.rand(z.shape[0], generator=gen, dtype=torch.float64).to("cuda") * 3.0
    w = torch.randn(z.shape[0], generator=gen, dtype=torch.float64).to("cuda")
    out = {}
    for dense_max in (10 ** 9, 0):
        m.eeq_dense_max = dense_max
        pos = pos0.clone().requires_grad_(True)
        c = cn.clone().requires_grad_(True)
        q = m.eeq_charges(z, pos, c, torch.tensor(0.5, dtype=torch.float64))
        gp, gc = torch.autograd.grad((q * w).sum(), (pos, c))
        out[dense_max] = (q.detach(), gp, gc)
    (qa, pa, ca), (qb, pb, cb) = out[10 ** 9], out[0]
    torch.testing.assert_close(qb, qa, rtol=1e-9, atol=1e-11)
    assert abs(float(qb.sum()) - 0.5) < 1e-10
    torch.testing.assert_close(pb, pa, rtol=1e-8, atol=1e-10)
    torch.testing.assert_close(cb, ca, rtol=1e-8, atol=1e-10)
