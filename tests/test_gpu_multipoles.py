"""Multipole real-space pair kernel against the PyTorch formulas (float64 on the GPU)."""
import pytest
import torch

from xnn_b200 import _ext
from xnn_b200.ffnn import multipoles as M

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_ext():
    if not _ext.cuda_available():
        pytest.fail(f"native extension not loaded: {_ext.error()}")


def _water(n=600):
    from xnn_b200.ffnn.water import multipole_water
    return multipole_water(n, seed=3, device="cuda")


@pytest.mark.parametrize("thole", [None, 0.39])
def test_pair_kernel_energy_and_gradients(thole, monkeypatch):
    w = _water()
    pairs = M.multipole_pairs(w["pos"], w["cell"], 7.0, w["molecule"])
    i, j, s, ex = pairs
    pos = w["pos"].clone().requires_grad_(True)
    d = w["d"].clone().requires_grad_(True)
    e_k = M.real_energy(pos, w["cell"], i, j, s, ex, w["q"], d, w["Q"], 0.4, pol=w["pol"], thole=thole)
    gp_k, gd_k = torch.autograd.grad(e_k, (pos, d))
    monkeypatch.setattr(M, "_kernel_ok", lambda: False)
    pos2 = w["pos"].clone().requires_grad_(True)
    d2 = w["d"].clone().requires_grad_(True)
    e_t = M.real_energy(pos2, w["cell"], i, j, s, ex, w["q"], d2, w["Q"], 0.4, pol=w["pol"], thole=thole)
    gp_t, gd_t = torch.autograd.grad(e_t, (pos2, d2))
    torch.testing.assert_close(e_k, e_t, rtol=1e-11, atol=1e-10)
    torch.testing.assert_close(gp_k, gp_t, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(gd_k, gd_t, rtol=1e-10, atol=1e-10)


def test_polarizable_evaluation_kernel_vs_torch(monkeypatch):
    w = _water(900)
    setup = M.EwaldSetup(alpha=0.4, cutoff=7.0, mesh=(48, 48, 48), order=5, fft_dtype=torch.float64)
    mod = M.PolarizableMultipoles(setup, tol_debye=1e-8, max_iter=200)
    a = mod(w["pos"], w["cell"], w["q"], w["d"], w["Q"], w["pol"], w["molecule"])
    monkeypatch.setattr(M, "_kernel_ok", lambda: False)
    b = mod(w["pos"], w["cell"], w["q"], w["d"], w["Q"], w["pol"], w["molecule"])
    torch.testing.assert_close(a["energy"], b["energy"], rtol=1e-10, atol=1e-8)
    torch.testing.assert_close(a["forces"], b["forces"], rtol=1e-7, atol=1e-8)
    torch.testing.assert_close(a["induced_dipoles"], b["induced_dipoles"], rtol=1e-7, atol=1e-9)


def test_spread_and_gather_kernels_match_torch(monkeypatch):
    w = _water(600)
    mesh, p = [40, 36, 32], 5
    pos = w["pos"].clone().requires_grad_(True)
    d = w["d"].clone().requires_grad_(True)
    grid_k = M.spread(pos, w["cell"], w["q"], d, w["Q"], mesh, p, out_dtype=torch.float32)
    phi = torch.randn(grid_k.shape, device="cuda", dtype=torch.float32)
    gp_k, gd_k = torch.autograd.grad((grid_k * phi).sum(), (pos, d))
    monkeypatch.setattr(M, "_kernel_ok", lambda: False)
    pos2 = w["pos"].clone().requires_grad_(True)
    d2 = w["d"].clone().requires_grad_(True)
    grid_t = M.spread(pos2, w["cell"], w["q"], d2, w["Q"], mesh, p)
    gp_t, gd_t = torch.autograd.grad((grid_t * phi.double()).sum(), (pos2, d2))
    torch.testing.assert_close(grid_k.double(), grid_t, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(gp_k, gp_t, rtol=1e-9, atol=1e-9)
    torch.testing.assert_close(gd_k, gd_t, rtol=1e-9, atol=1e-9)
    # a slab of planes
    g_slab = M.spread(w["pos"], w["cell"], w["q"], w["d"], w["Q"], mesh, p, z_range=(8, 19))
    monkeypatch.undo()
    g_slab_k = M.spread(w["pos"], w["cell"], w["q"], w["d"], w["Q"], mesh, p, z_range=(8, 19), out_dtype=torch.float32)
    torch.testing.assert_close(g_slab_k.double(), g_slab, rtol=1e-5, atol=1e-6)


def test_float32_mesh_evaluation_close_to_float64(monkeypatch):
    w = _water(900)
    kw = dict(alpha=0.4, cutoff=7.0, mesh=(48, 48, 48), order=5)
    a = M.PolarizableMultipoles(M.EwaldSetup(fft_dtype=torch.float32, **kw), tol_debye=1e-7, max_iter=200)(
        w["pos"], w["cell"], w["q"], w["d"], w["Q"], w["pol"], w["molecule"])
    b = M.PolarizableMultipoles(M.EwaldSetup(fft_dtype=torch.float64, **kw), tol_debye=1e-7, max_iter=200)(
        w["pos"], w["cell"], w["q"], w["d"], w["Q"], w["pol"], w["molecule"])
    torch.testing.assert_close(a["energy"], b["energy"], rtol=2e-6, atol=1e-4)
    torch.testing.assert_close(a["forces"], b["forces"], rtol=1e-3, atol=2e-4)
