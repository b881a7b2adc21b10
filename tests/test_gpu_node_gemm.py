"""Node-level tcgen05 products (``csrc/node_gemm.cu``) against float64 PyTorch references."""
import pytest
import torch

from xnn_b200.ops import node_gemm as NG

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(1e-30))


def test_species_sort_is_stable_grouping():
    g = torch.Generator(device="cuda").manual_seed(0)
    z = torch.randint(0, 7, (2303,), device="cuda", generator=g)
    perm, seg = NG.species_sort(z, 7)
    ref = torch.argsort(z, stable=True)
    assert torch.equal(perm.long(), ref)
    counts = torch.bincount(z, minlength=7)
    assert torch.equal(seg.long()[1:] - seg.long()[:-1], counts)


def test_node_mm_dense_grouped_and_two_sources():
    torch.manual_seed(1)
    dev = "cuda"
    N, C = 2203, 96
    z = torch.randint(0, 7, (N,), device=dev)
    perm, seg = NG.species_sort(z, 7)
    X = torch.randn(N, C, device=dev)
    X2 = torch.randn(N, C, device=dev)
    W = torch.randn(C, C, device=dev) / C ** 0.5
    Ws = torch.randn(7, C, C, device=dev) / C ** 0.5
    Wcat = torch.randn(2 * C, 64, device=dev) / C ** 0.5
    packed = NG.pack([W.t()] + [Ws[k] for k in range(7)] + [Wcat])
    Y = torch.empty(N, C, device=dev)
    Ysp = torch.zeros(N, C, device=dev)
    Ycat = torch.ones(N, 64, device=dev)
    probs = [NG.MM(X, W.t(), Y, packed[0])]
    probs += [NG.MM(X, Ws[k], Ysp, packed[1 + k], perm=perm, seg=seg[k:k + 2], rows=N) for k in range(7)]
    probs += [NG.MM(X, Wcat, Ycat, packed[8], X1=X2, accumulate=True)]
    NG.mm(probs)
    torch.cuda.synchronize()
    assert NG.status(torch.device(dev)) == 0
    Xd = X.double()
    assert _rel(Y, Xd @ W.double().t()) < 1e-5
    ref_sp = torch.einsum("nc,ncd->nd", Xd, Ws.double()[z])
    assert _rel(Ysp, ref_sp) < 1e-5
    ref_cat = 1.0 + torch.cat([Xd, X2.double()], 1) @ Wcat.double()
    assert _rel(Ycat, ref_cat) < 1e-5


def test_node_mmT_two_sets_and_segments():
    torch.manual_seed(2)
    dev = "cuda"
    N, C = 2203, 96
    z = torch.randint(0, 7, (N,), device=dev)
    perm, seg = NG.species_sort(z, 7)
    X, Xd_, D, Dd = (torch.randn(N, C, device=dev) for _ in range(4))
    Dn = torch.randn(N, 16, device=dev)
    out = torch.empty(C, C, device=dev)
    out16 = torch.empty(C, 16, device=dev)
    outs = torch.empty(7, C, C, device=dev)
    probs = [NG.MMT(X, D, out, X1=Xd_, D1=Dd, scale=0.5), NG.MMT(X, Dn, out16)]
    probs += [NG.MMT(X, D, outs[k], X1=Xd_, D1=Dd, perm=perm, seg=seg[k:k + 2], rows0=N, rows1=N) for k in range(7)]
    NG.mmT(probs)
    # the counters reset themselves: a second launch gives the same numbers
    out_again = torch.empty_like(out)
    NG.mmT([NG.MMT(X, D, out_again, X1=Xd_, D1=Dd, scale=0.5)])
    torch.cuda.synchronize()
    assert NG.status(torch.device(dev)) == 0
    ref = 0.5 * (X.double().t() @ D.double() + Xd_.double().t() @ Dd.double())
    assert _rel(out, ref) < 1e-5
    assert torch.equal(out, out_again)
    assert _rel(out16, X.double().t() @ Dn.double()) < 1e-5
    for k in range(7):
        m = z == k
        r = X.double()[m].t() @ D.double()[m] + Xd_.double()[m].t() @ Dd.double()[m]
        assert _rel(outs[k], r) < 1e-5, k
