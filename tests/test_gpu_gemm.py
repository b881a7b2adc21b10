"""tcgen05 3xTF32 GEMM against float64 products."""
import pytest
import torch

from xnn_b200.ops import gemm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,N", [(1000, 8, 64), (4097, 64, 64), (300, 64, 384), (1280, 384, 64),
                                   (129, 40, 192), (2048, 96, 96), (70000, 64, 384), (68000, 384, 64),
                                   (100000, 64, 64)])
def test_tf32x3_gemm_accuracy(M, K, N):
    X = torch.randn(M, K, device="cuda")
    W = torch.randn(K, N, device="cuda")
    assert gemm.supported(X, W)
    Y = gemm.mm_raw(X, W)
    torch.cuda.synchronize()
    assert gemm.tc_status(X.device) == 0
    ref = (X.double() @ W.double())
    err = (Y.double() - ref).abs().max() / ref.abs().max()
    # float32 accumulation over K terms; a single TF32 pass would be near 1e-3
    assert err < 1e-5, float(err)


def test_tf32x3_gemm_col_scale_and_strided_rows():
    X = torch.randn(500, 80, device="cuda")[:, :64]
    W = torch.randn(128, 64, device="cuda").t()      # a transposed view: packed without a copy
    s = torch.rand(128, device="cuda")
    Y = gemm.mm_raw(X, W, s)
    ref = (X.double() @ W.double()) * s.double()
    assert ((Y.double() - ref).abs().max() / ref.abs().max()) < 2e-6


@pytest.mark.parametrize("M,K1,N", [(70000, 64, 384), (5000, 8, 64), (1000, 64, 64), (33, 16, 32), (4096, 128, 96),
                                    (68000, 8, 64)])
def test_tf32x3_reduce_accuracy(M, K1, N):
    X = torch.randn(M, K1, device="cuda")
    D = torch.randn(M, N, device="cuda")
    assert gemm.reduce_supported(X, D)
    G = gemm.mm_t_raw(X, D)
    torch.cuda.synchronize()
    assert gemm.tc_status(X.device) == 0
    ref = X.double().t() @ D.double()
    err = (G.double() - ref).abs().max() / ref.abs().max()
    assert err < 1e-5, float(err)


@pytest.mark.parametrize("M,K,N", [(21570, 96, 96), (30000, 96, 672), (17000, 64, 16)])
def test_matmul_autograd_two_orders(M, K, N):
    """The differentiable tensor-core product against float64 autograd, first and second order."""
    from xnn_b200.ops import gemm
    g = torch.Generator(device="cuda").manual_seed(1)
    X = torch.randn(M, K, device="cuda", generator=g, requires_grad=True)
    W = torch.randn(K, N, device="cuda", generator=g, requires_grad=True) / K ** 0.5
    V = torch.randn(M, N, device="cuda", generator=g)
    Y = gemm.matmul(X, W)
    Xd, Wd = X.detach().double().requires_grad_(True), W.detach().double().requires_grad_(True)
    Yd = Xd @ Wd
    torch.testing.assert_close(Y.double(), Yd, rtol=1e-5, atol=1e-5)
    gX, gW = torch.autograd.grad((Y * V).sum(), (X, W), create_graph=True)
    gXd, gWd = torch.autograd.grad((Yd * V.double()).sum(), (Xd, Wd), create_graph=True)
    torch.testing.assert_close(gX.double(), gXd, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(gW.double(), gWd, rtol=1e-5, atol=1e-3)
    U = torch.randn_like(gX)
    h, = torch.autograd.grad((gX * U).sum(), W)
    hd, = torch.autograd.grad((gXd * U.double()).sum(), Wd)
    torch.testing.assert_close(h.double(), hd, rtol=1e-5, atol=1e-3)


@pytest.mark.parametrize("M,K,N", [(5000, 8, 64), (70001, 64, 64), (333, 64, 128)])
def test_fused_silu_epilogue(M, K, N):
    X = torch.randn(M, K, device="cuda")
    W = torch.randn(K, N, device="cuda") / K ** 0.5
    Y = gemm.mm_act(X, W, 1, 1.7)
    ref = 1.7 * torch.nn.functional.silu(X.double() @ W.double())
    assert ((Y.double() - ref).abs().max() / ref.abs().max()) < 1e-5


@pytest.mark.parametrize("M,K", [(5000, 8), (70001, 64), (257, 64)])
def test_fused_tangent_pair_epilogue(M, K):
    """``[c silu(a) | c silu'(a) a']`` from the block-diagonal product of ``[h | h']``."""
    H = 64
    X = torch.randn(M, 2 * K, device="cuda")
    W = torch.randn(K, H, device="cuda") / K ** 0.5
    Y = gemm.mm_act(X, torch.block_diag(W, W), 2, 1.3)
    a = X[:, :K].double() @ W.double()
    ad = X[:, K:].double() @ W.double()
    s = torch.sigmoid(a)
    ref = torch.cat([1.3 * a * s, 1.3 * s * (1 + a * (1 - s)) * ad], 1)
    assert ((Y.double() - ref).abs().max() / ref.abs().max()) < 1e-5


def test_fused_radial_network_matches_stages():
    """The MD radial network (value and tangent, activations fused) against the staged one."""
    from xnn_b200.models.mace import MACE
    from xnn_b200.ops import lean_conv
    from xnn_b200.ops.radial import RadialSpec, _eff, _forward
    torch.manual_seed(0)
    m = MACE(species=[1, 8], cutoff=4.5, num_channels=32, n_rbf=8, num_interactions=2, max_ell=3,
             correlation=3, avg_num_neighbors=30.0).cuda()
    blk, ef = m.interactions[0], m.edge_feat
    net = blk.conv_tp_weights
    spec = RadialSpec(net, None, ef.rbf.freqs, ef.rbf.norm, ef.cutoff, ef.envelope.p)
    We = _eff([layer.weight for layer in net], spec)
    r = 0.8 + 3.6 * torch.rand(50000, device="cuda")
    R0, Rd0 = _forward(r, We, spec)[:2]
    R1, Rd1 = lean_conv._primal_tangent(r, We, spec)
    R2 = lean_conv._primal(r, We, spec)
    for a, b in ((R1, R0), (Rd1, Rd0), (R2, R0)):
        assert ((a - b).abs().max() / b.abs().max()) < 1e-5


def test_reduction_with_wide_left_operand_swaps():
    """``X^T D`` with ``X`` wider than the reduction kernel takes runs as ``(D^T X)^T``."""
    g = torch.Generator(device="cuda").manual_seed(3)
    X = torch.randn(40000, 192, device="cuda", generator=g)
    D = torch.randn(40000, 64, device="cuda", generator=g)
    want = (X.double().t() @ D.double()).float()
    got = gemm.mm_t_raw(X, D)
    assert got.shape == (192, 64)
    torch.testing.assert_close(got, want, rtol=2e-5, atol=2e-3)
    got2 = gemm.matmul_t(X, D)
    torch.testing.assert_close(got2, want, rtol=2e-5, atol=2e-3)
