"""SchNet and PaiNN: the reference framework's own implementations (when installed) evaluate the
same state dict to the same energies and forces; symmetry and force consistency otherwise."""
import os
import sys

import pytest
import torch

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.painn import PaiNN
from xnn_b200.models.schnet import SchNet

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _ref_module(name):
    if not os.path.isdir(os.path.join(REF, "xnn")):
        pytest.skip("reference framework not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import importlib
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        return importlib.import_module(name)


def _batch(periodic=False):
    if periodic:
        ss = synthetic.triclinic_crystals(2, seed=5, labels=False)
        for s in ss:
            s["atomic_numbers"] = torch.full_like(s["atomic_numbers"], 8)
    else:
        ss = synthetic.organic_molecules(3, seed=2, labels=False)
    return collate([structure_to_graph(s, 5.0) for s in ss])


def _ref_graph(b):
    ad = _ref_module("xnn.common.data")
    g = ad.AtomicGraph(pos=b.pos.clone(), atomic_numbers=b.atomic_numbers, edge_index=b.edge_index,
                       cell_shifts=b.cell_shifts, batch=b.batch, n_atoms=b.n_atoms, cell=b.cell, pbc=b.pbc)
    return g


@pytest.mark.parametrize("family,kw", [
    ("schnet", dict(n_features=16, n_interactions=2, n_rbf=10, cutoff=5.0)),
    ("painn", dict(n_features=16, n_interactions=2, n_rbf=10, cutoff=5.0)),
])
@pytest.mark.parametrize("periodic", [False, True])
def test_matches_reference_implementation(family, kw, periodic):
    mod = _ref_module(f"xnn.gnn.models.{family}")
    ref_cls = mod.SchNet if family == "schnet" else mod.PaiNN
    torch.manual_seed(0)
    ref = ref_cls(**kw).double()
    mine = (SchNet if family == "schnet" else PaiNN)(**kw).double()
    missing, unexpected = mine.load_state_dict(ref.state_dict(), strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    outs = _ref_module("xnn.common.models.outputs")
    b = _batch(periodic)
    o_ref = outs.ForceStressOutput(ref, compute_stress=periodic)(_ref_graph(b))
    o = ForceStressOutput(mine, compute_stress=periodic)(b.clone())
    torch.testing.assert_close(o["energy"], o_ref["energy"], rtol=1e-11, atol=1e-11)
    torch.testing.assert_close(o["forces"], o_ref["forces"], rtol=1e-10, atol=1e-11)
    if periodic:
        torch.testing.assert_close(o["stress"], o_ref["stress"], rtol=1e-10, atol=1e-11)


@pytest.mark.parametrize("cls", [SchNet, PaiNN])
def test_invariance_and_finite_difference_forces(cls):
    torch.manual_seed(1)
    m = cls(n_features=8, n_interactions=2, n_rbf=6, cutoff=5.0)
    b = _batch()
    o = ForceStressOutput(m)(b.clone())
    q, _ = torch.linalg.qr(torch.randn(3, 3))
    b2 = b.clone()
    b2.pos = b.pos @ q.T + 1.3
    o2 = ForceStressOutput(m)(b2)
    torch.testing.assert_close(o2["energy"], o["energy"], rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(o2["forces"], o["forces"] @ q.T, rtol=1e-9, atol=1e-10)
    k, eps = 4, 1e-6
    bp, bm = b.clone(), b.clone()
    bp.pos = b.pos.clone(); bm.pos = b.pos.clone()
    bp.pos[k, 1] += eps
    bm.pos[k, 1] -= eps
    fd = -(m(bp)["energy"].sum() - m(bm)["energy"].sum()) / (2 * eps)
    torch.testing.assert_close(o["forces"][k, 1], fd, rtol=1e-6, atol=1e-8)
