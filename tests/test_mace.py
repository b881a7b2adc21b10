"""MACE: reference vs fused decomposition, symmetry, forces, stress, padding (CPU)."""
import math

import pytest
import torch

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput, build_model
from xnn_b200.models.mace import MACE
from xnn_b200.train.graphed import pad_graph

SPECIES = [1, 6, 7, 8, 9, 16, 17]


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _model(**kw):
    base = dict(species=SPECIES, cutoff=4.5, num_channels=8, n_rbf=8, num_interactions=2, max_ell=3,
                correlation=3, avg_num_neighbors=6.0)
    base.update(kw)
    return MACE(**base)


def _batch(n=3, seed=0):
    return collate([structure_to_graph(s, 4.5) for s in synthetic.organic_molecules(n, seed=seed)])


def _rot(seed=0):
    g = torch.Generator().manual_seed(seed)
    q, _ = torch.linalg.qr(torch.randn(3, 3, generator=g))
    return q * torch.sign(torch.linalg.det(q))


@pytest.mark.parametrize("first", ["RealAgnosticResidualInteractionBlock", "RealAgnosticInteractionBlock"])
@pytest.mark.parametrize("lmax,corr", [(3, 3), (2, 2), (1, 3)])
def test_fused_matches_reference(first, lmax, corr):
    m = _model(max_ell=lmax, correlation=corr, interaction_first=first)
    f = ForceStressOutput(m)
    b = _batch()
    m.use_fast = False
    o1 = f(b.clone())
    m.use_fast = True
    o2 = f(b.clone())
    torch.testing.assert_close(o1["energy"], o2["energy"], rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(o1["forces"], o2["forces"], rtol=1e-11, atol=1e-11)


@pytest.mark.parametrize("fast", [False, True])
def test_rotation_translation_invariance(fast):
    m = _model().set_use_fast(fast)
    f = ForceStressOutput(m)
    b = _batch()
    o = f(b.clone())
    R = _rot(3)
    b2 = b.clone()
    b2.pos = b2.pos @ R.T + torch.tensor([1.0, -2.0, 0.5])
    o2 = f(b2)
    torch.testing.assert_close(o["energy"], o2["energy"], rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(o["forces"] @ R.T, o2["forces"], rtol=1e-9, atol=1e-9)


def test_forces_finite_difference():
    m = _model()
    f = ForceStressOutput(m)
    s = synthetic.organic_molecules(1, seed=4)[0]
    g = structure_to_graph(s, 4.5)
    F = f(g.clone())["forces"]
    h = 1e-5
    for atom, comp in [(0, 0), (3, 1), (5, 2)]:
        gp, gm = g.clone(), g.clone()
        gp.pos[atom, comp] += h
        gm.pos[atom, comp] -= h
        ep = m(gp)["energy"].sum()
        em = m(gm)["energy"].sum()
        fd = -(ep - em).detach() / (2 * h)
        assert abs(float(fd) - float(F[atom, comp])) < 1e-6


def test_periodic_stress_matches_strain_derivative():
    m = _model(num_channels=4)
    f = ForceStressOutput(m, compute_stress=True)
    s = synthetic.triclinic_crystals(1, seed=2, n_min=8, n_max=12, labels=False)[0]
    s["atomic_numbers"] = torch.tensor([SPECIES[i % len(SPECIES)] for i in range(len(s["pos"]))])
    g = structure_to_graph(s, 4.5)
    out = f(g.clone())
    sig = out["stress"][0]
    vol = float(torch.linalg.det(g.cell[0]).abs())
    h = 1e-5
    for (i, j) in [(0, 0), (0, 1), (2, 2)]:
        eps = torch.zeros(3, 3)
        eps[i, j] = eps[j, i] = h / 2 if i != j else h
        def energy(e):
            gg = g.clone()
            gg.pos = g.pos + g.pos @ e
            gg.cell = g.cell + g.cell @ e
            return float(m(gg)["energy"].sum())
        de = (energy(eps) - energy(-eps)) / (2 * h)
        # a symmetric off-diagonal strain h/2 in (i, j) and (j, i) moves the energy by h * sigma_ij V
        assert abs(de / vol - float(sig[i, j])) < 1e-6


@pytest.mark.parametrize("fast", [False, True])
def test_padding_is_inert(fast):
    m = _model().set_use_fast(fast)
    f = ForceStressOutput(m)
    b = _batch(4, seed=7)
    p = pad_graph(b, b.num_nodes + 37, b.num_edges + 501, b.num_graphs + 3, cutoff=4.5)
    assert p.edge_order == "dst"
    assert bool((p.edge_index[1][1:] >= p.edge_index[1][:-1]).all())
    o = f(b.clone())
    op = f(p.clone())
    torch.testing.assert_close(o["energy"], op["energy"][: b.num_graphs])
    torch.testing.assert_close(o["forces"], op["forces"][: b.num_nodes])
    assert op["forces"][b.num_nodes:].abs().max() < 1e-12


def test_size_extensive_batching():
    m = _model()
    mols = synthetic.organic_molecules(3, seed=9)
    gs = [structure_to_graph(s, 4.5) for s in mols]
    eb = m(collate(gs))["energy"]
    es = torch.cat([m(g)["energy"] for g in gs])
    torch.testing.assert_close(eb, es)


def test_state_dict_layout_and_config():
    from xnn_b200.config import from_dict
    cfg = from_dict({"model": {"name": "mace", "cutoff": 4.5, "n_features": 16,
                               "extra": {"species": SPECIES, "correlation": 3}}})
    m = build_model(cfg)
    keys = m.state_dict().keys()
    for k in ["interactions.0.linear_up.weight", "interactions.0.conv_tp_weights.layer0.weight",
              "products.0.symmetric_contractions.contractions.0.weights.0",
              "products.0.symmetric_contractions.contractions.0.U_matrix_3",
              "interactions.0.skip_tp.weight", "readouts.1.linear_2.weight", "atom_ref.weight"]:
        assert k in keys
    assert m.products[0].symmetric_contractions.contractions[0].U_matrix_3.shape == (16, 16, 16, 23)
    assert math.isclose(m.receptive_field(), 9.0)


def test_edge_chunks_match_single_pass():
    m = _model().set_use_fast(True).eval()
    f = ForceStressOutput(m)
    b = _batch(4, seed=2)
    o1 = f(b.clone())
    m.edge_chunk = 37
    o2 = f(b.clone())
    torch.testing.assert_close(o1["energy"], o2["energy"], rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(o1["forces"], o2["forces"], rtol=1e-11, atol=1e-11)
