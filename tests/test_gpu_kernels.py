"""CUDA kernels against the PyTorch formulas of the same ops: values, first and second derivatives."""
import pytest
import torch

from xnn_b200 import _ext
from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.ops import mace_ops as K

pytestmark = pytest.mark.gpu


def _graph(n=6, cutoff=4.5, seed=0):
    mols = synthetic.organic_molecules(n, seed=seed, labels=False)
    return collate([structure_to_graph(s, cutoff) for s in mols])


def _check_derivs(fn_fast, fn_ref, inputs, rtol, atol, second=True):
    ins_f = [x.detach().clone().requires_grad_(True) for x in inputs]
    ins_r = [x.detach().clone().requires_grad_(True) for x in inputs]
    out_f = fn_fast(*ins_f)
    out_r = fn_ref(*ins_r)
    out_f = out_f if isinstance(out_f, tuple) else (out_f,)
    out_r = out_r if isinstance(out_r, tuple) else (out_r,)
    for a, b in zip(out_f, out_r):
        torch.testing.assert_close(a, b, rtol=rtol, atol=atol)
    cots = [torch.randn_like(o) for o in out_r]
    gf = torch.autograd.grad(out_f, ins_f, cots, create_graph=True, allow_unused=True)
    gr = torch.autograd.grad(out_r, ins_r, cots, create_graph=True, allow_unused=True)
    for a, b in zip(gf, gr):
        if b is None:
            continue
        torch.testing.assert_close(a, b, rtol=rtol, atol=atol)
    if not second:
        return
    vs = [torch.randn_like(g) if g is not None else None for g in gr]
    sf = sum((g * v).sum() for g, v in zip(gf, vs) if g is not None)
    sr = sum((g * v).sum() for g, v in zip(gr, vs) if g is not None)
    hf = torch.autograd.grad(sf, ins_f, allow_unused=True)
    hr = torch.autograd.grad(sr, ins_r, allow_unused=True)
    for a, b in zip(hf, hr):
        if b is None:
            continue
        assert a is not None
        torch.testing.assert_close(a, b, rtol=rtol, atol=atol)


@pytest.fixture(scope="module", autouse=True)
def _need_ext():
    if not _ext.cuda_available():
        pytest.fail(f"native extension not loaded: {_ext.error()}")


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-9), (torch.float32, 2e-4)])
@pytest.mark.parametrize("lmax", [1, 2, 3])
def test_edge_geometry(dtype, tol, lmax):
    g = _graph()
    vec = g.edge_vectors().to("cuda", dtype)
    freqs = (torch.pi * torch.arange(1, 9, dtype=dtype, device="cuda"))
    cfg = (lmax, freqs, (2 / 4.5) ** 0.5, 4.5, 5)
    _check_derivs(lambda v: K.edge_geometry(v, *cfg), lambda v: K.edge_features_torch(v, *cfg), [vec], tol, tol)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-9), (torch.float32, 5e-4)])
@pytest.mark.parametrize("P,C", [(4, 96), (3, 40), (2, 16), (4, 160)])
def test_conv(dtype, tol, P, C):
    g = _graph()
    dev = "cuda"
    ei = g.edge_index.to(dev)
    N, E = g.num_nodes, g.num_edges
    plan = K.EdgePlan.build(ei, N)
    x = torch.randn(N, C, dtype=dtype, device=dev)
    R = torch.randn(E, P, C, dtype=dtype, device=dev)
    Y = torch.randn(E, P * P, dtype=dtype, device=dev)
    _check_derivs(lambda a, b, c: K.conv(a, b, c, plan), lambda a, b, c: K.conv_torch(a, b, c, plan),
                  [x, R, Y], tol, tol)


def test_conv_unsorted_edges():
    g = _graph()
    dev = "cuda"
    perm = torch.randperm(g.num_edges)
    ei = g.edge_index[:, perm].to(dev)
    N, E, P, C = g.num_nodes, g.num_edges, 4, 32
    plan = K.EdgePlan.build(ei, N)
    assert plan.dst_perm is not None
    x = torch.randn(N, C, dtype=torch.float64, device=dev)
    R = torch.randn(E, P, C, dtype=torch.float64, device=dev)
    Y = torch.randn(E, P * P, dtype=torch.float64, device=dev)
    _check_derivs(lambda a, b, c: K.conv(a, b, c, plan), lambda a, b, c: K.conv_torch(a, b, c, plan),
                  [x, R, Y], 1e-9, 1e-9)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-9), (torch.float32, 5e-4)])
@pytest.mark.parametrize("lmax,corr", [(3, 3), (2, 3), (1, 2), (3, 1)])
def test_symmetric_contraction(dtype, tol, lmax, corr):
    dev = "cuda"
    N, C, n_el = 300, 40, 5
    D = (lmax + 1) ** 2
    Kn = K.num_invariants(lmax, corr)
    A = 0.5 * torch.randn(D, N, C, dtype=dtype, device=dev)
    W = torch.randn(n_el, Kn, C, dtype=dtype, device=dev)
    z = torch.randint(0, n_el, (N,), device=dev)
    _check_derivs(lambda a, w: K.symmetric_contraction(a, w, z, lmax, corr),
                  lambda a, w: K.symmetric_contraction_torch(a, w, z, lmax, corr), [A, W], tol, tol)


def test_neighbor_list_cuda_matches_cpu():
    from xnn_b200.data.neighborlist import build_neighbor_list
    for s in synthetic.triclinic_crystals(2, seed=5, labels=False) + [synthetic.water_box(6000)]:
        a = build_neighbor_list(s["pos"], 5.0, s["cell"], s["pbc"], engine="native")
        b = build_neighbor_list(s["pos"].cuda(), 5.0, s["cell"].cuda(), s["pbc"], engine="native")
        ka = torch.unique(torch.cat([a[0].T, a[1]], 1), dim=0)
        kb = torch.unique(torch.cat([b[0].T.cpu(), b[1].cpu()], 1), dim=0)
        assert torch.equal(ka, kb)


def test_neighbor_list_warp_kernel_matches_thread_kernel(monkeypatch):
    """The warp-per-receiver search gives the thread-per-receiver kernel's edges in the same order
    (and a receiver range its share)."""
    from xnn_b200.data.neighborlist import build_neighbor_list
    for s in synthetic.triclinic_crystals(2, seed=7, labels=False) + [synthetic.water_box(6000)]:
        args = (s["pos"].cuda(), 5.0, s["cell"].cuda(), s["pbc"])
        a = build_neighbor_list(*args, engine="native")
        r = build_neighbor_list(*args, engine="native", receivers=(7, s["pos"].shape[0] // 2))
        monkeypatch.setenv("XNN_B200_NB_THREAD", "1")
        b = build_neighbor_list(*args, engine="native")
        rb = build_neighbor_list(*args, engine="native", receivers=(7, s["pos"].shape[0] // 2))
        monkeypatch.delenv("XNN_B200_NB_THREAD")
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
        assert torch.equal(r[0], rb[0]) and torch.equal(r[1], rb[1])


def test_schnet_cfconv_kernel_matches_torch_path():
    from xnn_b200.models import ForceStressOutput
    from xnn_b200.models.schnet import SchNet
    torch.manual_seed(0)
    m = SchNet(n_features=64, n_interactions=3, n_rbf=20, cutoff=5.0).cuda().double()
    g = _graph(n=8, cutoff=5.0).to("cuda")
    g.pos = g.pos.double()
    o_fast = ForceStressOutput(m.set_use_fast(True))(g.clone())
    o_ref = ForceStressOutput(m.set_use_fast(False))(g.clone())
    torch.testing.assert_close(o_fast["energy"], o_ref["energy"], rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(o_fast["forces"], o_ref["forces"], rtol=1e-9, atol=1e-10)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-10), (torch.float32, 1e-4)])
@pytest.mark.parametrize("C", [96, 160])
def test_sender_rows_match_scatter(dtype, tol, C):
    """Per-edge sender terms of the edge kernel, summed per sender, equal the scatter kernel's sums."""
    g = _graph()
    ei = g.edge_index.to("cuda")
    N, E, P = g.num_nodes, g.num_edges, 4
    plan = K.EdgePlan.build(ei, N)
    ops = _ext.ops()
    G = torch.randn(P * P, N, C, dtype=dtype, device="cuda")
    x = torch.randn(N, C, dtype=dtype, device="cuda")
    R = torch.randn(E, P, C, dtype=dtype, device="cuda")
    Rd = torch.randn(E, P, C, dtype=dtype, device="cuda")
    Y = torch.randn(E, P * P, dtype=dtype, device="cuda")
    g_r, gY, T1, _, _ = ops.conv_edge(N, C, P, E, plan.dst_ptr, plan.src32, plan.dst_perm, G, [Y], [x], [True],
                                      True, [x], [R], Rd)
    ref = ops.conv_scatter(plan.n_senders, C, P, plan.src_ptr, plan.src_perm, [R], [T1])
    g_r2, gY2, _, _, v = ops.conv_edge(N, C, P, E, plan.dst_ptr, plan.src32, plan.dst_perm, G, [Y], [x], [False],
                                       True, [x], [R], Rd, R)
    got = ops.conv_sender_sum(plan.n_senders, plan.src_ptr, plan.src_perm, v)
    torch.testing.assert_close(got, ref, rtol=tol, atol=tol)
    torch.testing.assert_close(g_r2, g_r, rtol=tol, atol=tol)
    torch.testing.assert_close(gY2, gY, rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-10), (torch.float32, 1e-4)])
@pytest.mark.parametrize("P,C", [(4, 96), (3, 40), (4, 160), (2, 128)])
def test_force_kernel_matches_formulas(dtype, tol, P, C):
    """The force-pass kernel (g_r, gY, sender terms) against the PyTorch formulas, fp64 reference."""
    g = _graph()
    ei = g.edge_index
    ei = ei[:, torch.argsort(ei[1], stable=True)].to("cuda")
    N, E = g.num_nodes, ei.shape[1]
    plan = K.EdgePlan.build(ei, N, assume_dst_sorted=True)
    assert plan.dst_perm is None
    G = torch.randn(P * P, N, C, dtype=torch.float64, device="cuda")
    x = torch.randn(N, C, dtype=torch.float64, device="cuda")
    R = torch.randn(E, P, C, dtype=torch.float64, device="cuda")
    Rd = torch.randn(E, P, C, dtype=torch.float64, device="cuda")
    Y = torch.randn(E, P * P, dtype=torch.float64, device="cuda")
    src, dst = ei[0], ei[1]
    lidx = torch.tensor([l for l in range(P) for _ in range(2 * l + 1)], device="cuda")
    Gd = G[:, dst].permute(1, 0, 2)                                   # (E, D, C)
    T = torch.zeros(E, P, C, dtype=torch.float64, device="cuda").index_add_(1, lidx, Gd * Y[:, :, None])
    xs = x[src]
    ref_gr = (xs[:, None, :] * T * Rd).sum((1, 2))
    ref_gY = (Gd * R[:, lidx, :] * xs[:, None, :]).sum(-1)
    ref_gxe = (T * R).sum(1)
    cast = [t.to(dtype) for t in (G, Y, x, R, Rd)]
    g_r, gY, gxe = _ext.ops().conv_force(N, C, P, E, plan.dst_ptr, plan.src32, *cast)
    torch.testing.assert_close(g_r.double(), ref_gr, rtol=tol, atol=tol * 10)
    torch.testing.assert_close(gY.double(), ref_gY, rtol=tol, atol=tol * 10)
    torch.testing.assert_close(gxe.double(), ref_gxe, rtol=tol, atol=tol * 10)


def test_lean_chunks_match_single_pass():
    """The chunked force pass (radial network recomputed per chunk) against the unchunked one."""
    from xnn_b200.models import ForceStressOutput
    from xnn_b200.models.mace import MACE
    torch.manual_seed(0)
    m = MACE(species=[1, 6, 7, 8], cutoff=4.5, num_channels=32, max_ell=3, correlation=3, num_interactions=2,
             hidden_irreps="32x0e").double().cuda().eval().set_use_fast(True)
    f = ForceStressOutput(m)
    b = _graph(n=5, seed=3).to("cuda")
    b.pos = b.pos.double()
    m.edge_chunk = None
    o1 = f(b.clone())
    m.edge_chunk = 301
    o2 = f(b.clone())
    torch.testing.assert_close(o2["energy"], o1["energy"], rtol=1e-11, atol=1e-11)
    torch.testing.assert_close(o2["forces"], o1["forces"], rtol=1e-10, atol=1e-10)
