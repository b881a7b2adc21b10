"""TensorNet compact messages: the three linear forms against dense formulas, gradients to second
order (gradcheck / gradgradcheck in float64), and on a GPU the kernels against the CPU formulas."""
import pytest
import torch

from xnn_b200.ops import tensornet_ops as T


def _case(n=7, E=23, F=5, seed=0, device="cpu", dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n, (E,), generator=g)
    dst = torch.randint(0, n, (E,), generator=g)
    a = torch.randn(E, 3, F, generator=g, dtype=dtype)
    x = torch.randn(n, 10, F, generator=g, dtype=dtype)
    y = torch.randn(n, 10, F, generator=g, dtype=dtype)
    plan = T.TensorPlan.build(src.to(device), dst.to(device), n)
    return plan, a.to(device), x.to(device), y.to(device), src, dst


def test_forms_match_dense_sums():
    plan, a, x, y, src, dst = _case()
    grp = torch.tensor(T.GROUP)
    m = T.messages(a, x, plan)
    want = torch.zeros_like(m)
    for p in range(src.shape[0]):
        want[dst[p]] += a[p, grp] * x[src[p]]
    torch.testing.assert_close(m, want)
    mt = T._MT.apply(a, y, plan)
    want = torch.zeros_like(mt)
    for p in range(src.shape[0]):
        want[src[p]] += a[p, grp] * y[dst[p]]
    torch.testing.assert_close(mt, want)
    d = T._D.apply(y, x, plan)
    prod = y[dst] * x[src]
    torch.testing.assert_close(d, torch.stack([prod[:, 0], prod[:, 1:4].sum(1), prod[:, 4:].sum(1)], 1))


def test_second_order_gradients():
    plan, a, x, y, _, _ = _case(n=4, E=6, F=2)
    for fn, args in ((T._M.apply, (a, x)), (T._MT.apply, (a, y)), (T._D.apply, (y, x))):
        inp = tuple(t.clone().requires_grad_(True) for t in args)
        f = lambda u, v: fn(u, v, plan)  # noqa: E731
        assert torch.autograd.gradcheck(f, inp)
        assert torch.autograd.gradgradcheck(f, inp)


def test_embedding_forms_and_second_order():
    plan, a, x, y, src, dst = _case(n=6, E=15, F=3, seed=2)
    geo = T.geometry_rows(torch.nn.functional.normalize(torch.randn(15, 3, dtype=torch.float64), dim=-1))
    grp = torch.tensor(T.GROUP)
    out = T.embedding(a, geo, plan)
    want = torch.zeros_like(out)
    for p in range(15):
        want[dst[p]] += a[p, grp] * geo[p][:, None]
    torch.testing.assert_close(out, want)
    plan, a, x, y, _, _ = _case(n=4, E=6, F=2, seed=5)
    geo = torch.randn(6, 10, dtype=torch.float64)
    for fn, args in ((T._Em.apply, (a, geo)), (T._Ea.apply, (y, geo)), (T._Eg.apply, (a, y))):
        inp = tuple(t.clone().requires_grad_(True) for t in args)
        f = lambda u, v: fn(u, v, plan)  # noqa: E731
        assert torch.autograd.gradcheck(f, inp)
        assert torch.autograd.gradgradcheck(f, inp)


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_matmul3_and_its_derivatives(ta, tb):
    g = torch.Generator().manual_seed(7)
    A = torch.randn(3, 3, 3, 2, generator=g, dtype=torch.float64, requires_grad=True)
    B = torch.randn(3, 3, 3, 2, generator=g, dtype=torch.float64, requires_grad=True)
    a = A.permute(0, 3, 1, 2)
    b = B.permute(0, 3, 1, 2)
    want = (a.transpose(-1, -2) if ta else a) @ (b.transpose(-1, -2) if tb else b)
    torch.testing.assert_close(T.matmul3(A, B, ta, tb), want.permute(0, 2, 3, 1))
    f = lambda u, v: T.matmul3(u, v, ta, tb)  # noqa: E731
    assert torch.autograd.gradcheck(f, (A, B))
    assert torch.autograd.gradgradcheck(f, (A, B))


@pytest.mark.gpu
def test_matmul3_kernel_matches_cpu():
    g = torch.Generator().manual_seed(8)
    for ta, tb in ((False, False), (True, False), (False, True), (True, True)):
        A = torch.randn(50, 3, 3, 64, generator=g)
        B = torch.randn(50, 3, 3, 64, generator=g)
        torch.testing.assert_close(T.matmul3(A.cuda(), B.cuda(), ta, tb).cpu(), T.matmul3(A, B, ta, tb),
                                   rtol=1e-5, atol=1e-5)


def test_compact_round_trip():
    s = torch.randn(4, 3, 3, 2, dtype=torch.float64)
    sym = 0.5 * (s + s.transpose(1, 2))
    c = T.to_compact(torch.randn(4, 2, dtype=torch.float64), torch.randn(4, 3, 2, dtype=torch.float64), sym)
    torch.testing.assert_close(T.sym_from_compact(c[:, 4:]), sym)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,F,tol", [(torch.float64, 64, 1e-12), (torch.float32, 64, 1e-5),
                                         (torch.float32, 128, 1e-5), (torch.float64, 20, 1e-12)])
def test_kernels_match_cpu(dtype, F, tol):
    plan_c, a, x, y, src, dst = _case(n=300, E=9000, F=F, seed=3, dtype=dtype)
    plan_g = T.TensorPlan.build(src.cuda(), dst.cuda(), 300)
    ac, xc, yc = (t.clone().requires_grad_(True) for t in (a, x, y))
    ag, xg, yg = (t.cuda().requires_grad_(True) for t in (a, x, y))
    # forward, first and second derivatives through the message sum (the force-loss pattern)
    def chain(aa, xx, yy, plan):
        m = T.messages(aa, xx, plan)
        (ga, gx) = torch.autograd.grad((m * yy).sum(), (aa, xx), create_graph=True)
        return m, ga, gx, (ga * ga).sum() + (gx * gx).sum()
    mc, gac, gxc, lc = chain(ac, xc, yc, plan_c)
    mg, gag, gxg, lg = chain(ag, xg, yg, plan_g)
    for u, v in ((mc, mg), (gac, gag), (gxc, gxg)):
        torch.testing.assert_close(v.cpu(), u.detach(), rtol=tol, atol=tol)
    hc = torch.autograd.grad(lc, (ac, xc, yc))
    hg = torch.autograd.grad(lg, (ag, xg, yg))
    for u, v in zip(hc, hg):
        torch.testing.assert_close(v.cpu(), u, rtol=tol * 10, atol=tol * 10)
    # the embedding forms through the same pattern (geometry rows carry the force path)
    geo = T.geometry_rows(torch.nn.functional.normalize(torch.randn(9000, 3, dtype=dtype), dim=-1))
    gc = geo.clone().requires_grad_(True)
    gg = geo.cuda().requires_grad_(True)
    ac2, ag2 = a.clone().requires_grad_(True), a.cuda().requires_grad_(True)

    def chain_e(aa, ge, yy, plan):
        m = T.embedding(aa, ge, plan)
        (ga, gq) = torch.autograd.grad((m * yy).sum(), (aa, ge), create_graph=True)
        return m, ga, gq, (ga * ga).sum() + (gq * gq).sum()
    outc = chain_e(ac2, gc, y, plan_c)
    outg = chain_e(ag2, gg, y.cuda(), plan_g)
    for u, v in zip(outc[:3], outg[:3]):
        torch.testing.assert_close(v.detach().cpu(), u.detach(), rtol=tol, atol=tol)
    hc = torch.autograd.grad(outc[3], (ac2, gc))
    hg = torch.autograd.grad(outg[3], (ag2, gg))
    for u, v in zip(hc, hg):
        torch.testing.assert_close(v.cpu(), u, rtol=tol * 10, atol=tol * 10)
