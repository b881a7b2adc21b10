"""Model families against the reference framework's own implementations: the same state dict
gives the same energies, forces and stress (float64)."""
import pytest
import torch

from ref_oracle import batch, compare, load_same_weights, ref_module


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _pair(mod_name, ref_cls, mine_cls, seed=0, **kw):
    mod = ref_module(mod_name)
    torch.manual_seed(seed)
    ref = getattr(mod, ref_cls)(**kw).double()
    mine = mine_cls(**kw).double()
    load_same_weights(mine, ref)
    return mine, ref


@pytest.mark.parametrize("readout", ["mlp", "gated"])
@pytest.mark.parametrize("periodic", [False, True])
def test_tensornet(readout, periodic):
    from xnn_b200.models.tensornet import TensorNet
    mine, ref = _pair("xnn.gnn.models.tensornet", "TensorNet", TensorNet, n_features=8, n_interactions=2, n_rbf=8,
                      cutoff=5.0, readout=readout)
    compare(mine, ref, batch(periodic), periodic)


@pytest.mark.parametrize("hardness", ["element", "environment"])
@pytest.mark.parametrize("periodic", [False, True])
def test_qet(hardness, periodic):
    from xnn_b200.models.qet import QET
    mine, ref = _pair("xnn.gnn.models.qet", "QET", QET, n_features=8, n_interactions=2, n_rbf=8, cutoff=5.0,
                      hardness=hardness)
    b = batch(periodic)
    extra = {"total_charge": torch.tensor([1.0, -1.0] + ([0.0] if not periodic else []))}
    compare(mine, ref, b, periodic, keys=("charges",), **extra)
