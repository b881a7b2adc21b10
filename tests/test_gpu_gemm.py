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
