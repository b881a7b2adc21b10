"""Hessians (fused and reference MACE paths agree; symmetric; match finite differences of forces)
and harmonic analysis of a diatomic (the analytic harmonic frequency)."""
import math

import pytest
import torch

from xnn_b200.data import structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.mace import MACE
from xnn_b200.models.vibrations import hessian, hessian_vector_product, harmonic_analysis, WAVENUMBER


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def test_hessian_symmetric_and_matches_force_differences():
    torch.manual_seed(0)
    m = MACE(species=[1, 6, 7, 8, 9, 16, 17], cutoff=4.5, num_channels=8, n_rbf=6, num_interactions=2,
             max_ell=2, correlation=2, avg_num_neighbors=5.0)
    s = synthetic.organic_molecules(1, seed=3, labels=False)[0]
    s["pos"], s["atomic_numbers"] = s["pos"][:8], s["atomic_numbers"][:8]
    g = structure_to_graph(s, 4.5)
    (H,) = hessian(m.set_use_fast(True), g)
    (H_ref,) = hessian(m.set_use_fast(False), g)
    torch.testing.assert_close(H, H_ref, rtol=1e-9, atol=1e-10)
    torch.testing.assert_close(H, H.t(), rtol=1e-9, atol=1e-10)
    v = torch.randn(8, 3)
    torch.testing.assert_close(hessian_vector_product(m, g, v).reshape(-1), H @ v.reshape(-1), rtol=1e-9, atol=1e-10)
    eps = 1e-5
    f = ForceStressOutput(m)
    gp, gm = g.clone(), g.clone()
    gp.pos = g.pos.clone(); gm.pos = g.pos.clone()
    gp.pos[2, 1] += eps
    gm.pos[2, 1] -= eps
    col = -(f(gp)["forces"] - f(gm)["forces"]).reshape(-1) / (2 * eps)
    torch.testing.assert_close(H[:, 7], col, rtol=1e-6, atol=1e-7)


def test_harmonic_analysis_of_a_diatomic():
    k, m1, m2 = 5.0, 1.008, 15.999
    pos = torch.tensor([[0.0, 0.0, 0.0], [0.0, 0.0, 1.0]])
    H = torch.zeros(6, 6)
    for a, b, sgn in ((0, 0, 1), (1, 1, 1), (0, 1, -1), (1, 0, -1)):
        H[3 * a + 2, 3 * b + 2] = sgn * k
    out = harmonic_analysis(H, pos, masses=torch.tensor([m1, m2]))
    mu = m1 * m2 / (m1 + m2)
    assert out["linear"] and out["frequencies"].shape == (1,)
    assert abs(float(out["frequencies"][0]) - math.sqrt(k / mu) * WAVENUMBER) < 1e-6
