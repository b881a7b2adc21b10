"""The native D3 two-body passes (CUDA kernels; OpenMP twin on the CPU) against the PyTorch D3:
per-atom energies, coordination numbers, features and forces by autograd, rational and zero
damping, molecules and a periodic cell."""
import pytest
import torch

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.d3 import D3Dispersion


def _batch(periodic, device="cpu"):
    if periodic:
        s = synthetic.triclinic_crystals(2, seed=5, n_min=12, n_max=24, z_max=36)
    else:
        s = synthetic.organic_molecules(3, seed=6, n_min=8, n_max=20)
    b = collate([structure_to_graph(x, 12.0) for x in s]).to(device)
    b.pos = b.pos.double()
    return b


def _run(kernels, damping, periodic, device="cpu", switch=0.0):
    torch.set_default_dtype(torch.float64)
    try:
        pot = D3Dispersion(damping=damping, cutoff_pair=12.0, cutoff_cn=10.0, switch_width_pair=switch).to(device).eval()
        pot.d3.use_kernels = kernels
        assert pot.d3.kernels_usable(torch.zeros(1, 3, device=device)) == kernels
        out = ForceStressOutput(pot).eval()(_batch(periodic, device))
        return {k: out[k].detach().cpu() for k in ("energy", "forces", "node_energy", "coordination_numbers",
                                                   "node_features")}
    finally:
        torch.set_default_dtype(torch.float32)


@pytest.mark.parametrize("damping", ["bj", "zero"])
@pytest.mark.parametrize("periodic", [False, True])
def test_native_two_body_matches_torch(damping, periodic):
    a = _run(True, damping, periodic, switch=1.5 if periodic else 0.0)
    b = _run(False, damping, periodic, switch=1.5 if periodic else 0.0)
    for k in a:
        torch.testing.assert_close(a[k], b[k], rtol=1e-10, atol=1e-12, msg=k)


@pytest.mark.gpu
@pytest.mark.parametrize("damping", ["bj", "zero"])
def test_cuda_two_body_matches_torch(damping):
    a = _run(True, damping, True, device="cuda", switch=1.5)
    b = _run(False, damping, True, device="cpu", switch=1.5)
    for k in a:
        torch.testing.assert_close(a[k], b[k], rtol=1e-10, atol=1e-12, msg=k)
