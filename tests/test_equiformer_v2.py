"""EquiformerV2 pieces against closed forms: the S2 grid transforms invert each other and sample
the harmonics; edge frames map edges onto +y and their Wigner matrices are orthogonal
representations; the gated model is rotation invariant with equivariant forces."""
import math

import pytest
import torch

from xnn_b200.data import collate, structure_to_graph
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.equiformer_v2 import EdgeFrames, EquiformerV2, edge_rotation
from xnn_b200.o3 import FromS2Grid, ToS2Grid, spherical_harmonics
from xnn_b200.o3._s2grid import grid_points, s2_grid


@pytest.mark.parametrize("norm", ["component", "norm", "integral"])
def test_s2_grid_round_trip(norm):
    to, fr = ToS2Grid(3, (8, 9), norm, dtype=torch.float64), FromS2Grid((8, 9), 3, norm, dtype=torch.float64)
    x = torch.randn(4, 16, dtype=torch.float64)
    torch.testing.assert_close(fr(to(x)), x, rtol=1e-12, atol=1e-12)


def test_s2_grid_samples_harmonics():
    b, a = s2_grid(6, 7)
    y = spherical_harmonics([0, 1, 2], grid_points(b, a), normalization="integral")
    x = torch.randn(9, dtype=torch.float64)
    torch.testing.assert_close(ToS2Grid(2, (6, 7), "integral", dtype=torch.float64)(x), y @ x, rtol=1e-12, atol=1e-12)


def test_edge_frames():
    vec = torch.randn(20, 3, dtype=torch.float64)
    vec[0] = torch.tensor([0.0, -2.0, 0.0], dtype=torch.float64)       # south pole
    rot = edge_rotation(vec)
    unit = vec / vec.norm(dim=1, keepdim=True)
    torch.testing.assert_close(torch.einsum("eij,ej->ei", rot, unit), torch.tensor([0.0, 1.0, 0.0]).double().expand(20, 3))
    torch.testing.assert_close(torch.linalg.det(rot), torch.ones(20, dtype=torch.float64))
    for d in EdgeFrames(3)(vec):
        eye = torch.eye(d.shape[1], dtype=torch.float64).expand_as(d)
        torch.testing.assert_close(d @ d.transpose(1, 2), eye, rtol=1e-12, atol=1e-12)


def _rotation(seed=3):
    q, _ = torch.linalg.qr(torch.randn(3, 3, generator=torch.Generator().manual_seed(seed), dtype=torch.float64))
    return q * torch.sign(torch.linalg.det(q))


@pytest.mark.parametrize("mmax", [2, 1])
def test_rotation_invariance(mmax):
    torch.manual_seed(0)
    model = EquiformerV2(n_features=8, n_interactions=2, cutoff=4.0, n_rbf=8, l_max=2, m_max=mmax, num_heads=2,
                         attn_hidden_channels=6, attn_alpha_channels=4, attn_value_channels=3, ffn_hidden_channels=8,
                         edge_channels=8, activation="gate", use_grid_mlp=False, norm_type="rms_norm_sh").double()
    pos = torch.randn(7, 3, dtype=torch.float64) * 1.3
    z = torch.tensor([6, 1, 1, 8, 7, 1, 6])
    R = _rotation()
    out = []
    for p in (pos, pos @ R.T):
        g = collate([structure_to_graph({"pos": p, "atomic_numbers": z}, 4.0)])
        out.append(ForceStressOutput(model)(g))
    torch.testing.assert_close(out[1]["energy"], out[0]["energy"], rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(out[1]["forces"], out[0]["forces"] @ R.T, rtol=1e-9, atol=1e-10)
