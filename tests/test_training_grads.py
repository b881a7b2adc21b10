"""Force-loss parameter gradients: fused decomposition (with the pass flags) vs the reference path."""
import pytest
import torch

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.mace import MACE
from xnn_b200.ops.modes import params_only


def _loss_grads(model, batch, flags: bool):
    f = ForceStressOutput(model).train()
    out = f(batch.clone())
    loss = ((out["energy"] - batch.energy) ** 2).mean() + 10 * ((out["forces"] - batch.forces) ** 2).mean()
    params = [p for p in model.parameters() if p.requires_grad]
    if flags:
        with params_only():
            g = torch.autograd.grad(loss, params, allow_unused=True)
    else:
        g = torch.autograd.grad(loss, params, allow_unused=True)
    return loss.detach(), g


@pytest.mark.parametrize("device,dtype,tol", [("cpu", torch.float64, 1e-8),
                                              pytest.param("cuda", torch.float64, 1e-8, marks=pytest.mark.gpu),
                                              pytest.param("cuda", torch.float32, 2e-3, marks=pytest.mark.gpu)])
def test_force_loss_gradients_match_reference(device, dtype, tol):
    torch.set_default_dtype(dtype)
    try:
        torch.manual_seed(1)
        m = MACE(species=[1, 6, 7, 8, 9, 16, 17], cutoff=4.5, num_channels=8, n_rbf=8, num_interactions=2,
                 max_ell=3, correlation=3, avg_num_neighbors=8.0).to(device)
        b = collate([structure_to_graph(s, 4.5) for s in synthetic.organic_molecules(3, seed=2)]).to(device)
        m.use_fast = False
        l1, g1 = _loss_grads(m, b, flags=False)
        m.use_fast = True
        l2, g2 = _loss_grads(m, b, flags=True)
        torch.testing.assert_close(l1, l2, rtol=tol, atol=tol * 1e-2)
        for a, c in zip(g1, g2):
            if a is None:
                assert c is None or c.abs().max() == 0
                continue
            scale = float(a.abs().max()) + 1e-30
            assert float((a - c).abs().max()) <= tol * scale + 1e-12
    finally:
        torch.set_default_dtype(torch.float32)
