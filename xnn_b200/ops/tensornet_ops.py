"""TensorNet messages on compact tensor rows, differentiable to any order.

An atom's tensor features are ten rows of ``F`` channels, ``x = [I, v_x, v_y, v_z, S_xx, S_xy,
S_xz, S_yy, S_yz, S_zz]`` (scalar, axial vector of the skew part, distinct entries of the
symmetric part), and a pair's filters three rows ``a = [a_I, a_A, a_S]``. The message sum of a
layer (reference: ``src/xnn/gnn/models/tensornet.py:317-368`` gathers the neighbours' parts to
the pairs, scales them and sums them onto the centres; the fused path of
``src/xnn/gnn/fast/tensornet_kernels.py:31-140`` does it in one kernel) is

    ``M(a, x)[i, c] = sum_{pairs j -> i} a[p, g(c)] * x[j, c]``    (``g``: 0 | 1,1,1 | 2 x 6)

and its two adjoints are of the same kind:

    ``M^T(a, y)[j, c] = sum_{pairs j -> i} a[p, g(c)] * y[i, c]``  (the sum over senders)
    ``D(y, x)[p, g]   = sum_{c in g} y[i, c] * x[j, c]``           (per pair)

``d M / d a = D``, ``d M / d x = M^T``, ``d M^T / d a = D`` (roles swapped), ``d M^T / d y = M``,
``d D / d y = M``, ``d D / d x = M^T``: three autograd functions whose backward passes call each
other differentiate to any order, each on one sm_100a kernel (``csrc/tensornet.cu``) with
nothing pair-sized beyond the filters and their gradients. The embedding is the same kind of
sum with per-pair geometry rows ``geo = [1, u, u u^T]`` in place of the neighbour's features
(``Em``, with adjoints ``Ea`` in the pair parts and ``Eg`` in the geometry). On the CPU the same
functions run their PyTorch formulas, and so do they on the GPU inside :func:`kernels_enabled`
``(False)`` (the model's ``use_fast=False``); each function's backward pass takes the forward
pass's choice.
"""
from __future__ import annotations

import contextlib
import functools
import threading
from dataclasses import dataclass
from typing import Optional

import torch
from torch import Tensor

from .. import _ext

GROUP = (0, 1, 1, 1, 2, 2, 2, 2, 2, 2)

_MODE = threading.local()


def _allowed() -> bool:
    return getattr(_MODE, "on", True)


@contextlib.contextmanager
def kernels_enabled(on: bool):
    """Within the block the functions here use their kernels (``True``) or formulas (``False``)."""
    prev = _allowed()
    _MODE.on = bool(on)
    try:
        yield
    finally:
        _MODE.on = prev


def _records_mode(fwd):
    @functools.wraps(fwd)
    def run(ctx, *args):
        ctx.kernels_on = _allowed()
        return fwd(ctx, *args)
    return run


def _keeps_mode(bwd):
    @functools.wraps(bwd)
    def run(ctx, *grads):
        with kernels_enabled(ctx.kernels_on):
            return bwd(ctx, *grads)
    return run


@dataclass
class TensorPlan:
    """Pairs ``src -> dst`` of ``n`` atoms with both CSR orderings (receivers and senders)."""
    src: Tensor
    dst: Tensor
    n: int
    dst_ptr: Tensor
    dst_order: Tensor
    src_ptr: Tensor
    src_order: Tensor

    @classmethod
    def build(cls, src: Tensor, dst: Tensor, n: int) -> "TensorPlan":
        src, dst = src.long().contiguous(), dst.long().contiguous()

        def csr(key):
            order = torch.sort(key, stable=True)[1]
            counts = torch.bincount(key, minlength=n)
            ptr = torch.zeros(n + 1, dtype=torch.long, device=key.device)
            ptr[1:] = torch.cumsum(counts, 0)
            return ptr, order

        dp, do = csr(dst)
        sp, so = csr(src)
        return cls(src, dst, n, dp, do, sp, so)


def _kernels(t: Tensor) -> bool:
    if not _allowed() or not t.is_cuda or t.dtype not in (torch.float32, torch.float64) or t.shape[-1] > 128:
        return False
    if not hasattr(_ext.ops(), "tn_gather"):
        raise RuntimeError("xnn_b200 extension without the TensorNet kernels: rebuild it (xnn_b200.build)")
    return True


def _expand(a: Tensor) -> Tensor:
    """``(E, 3, F)`` filters to ``(E, 10, F)`` per row."""
    return torch.cat([a[:, 0:1], a[:, 1:2].expand(-1, 3, -1), a[:, 2:3].expand(-1, 6, -1)], 1)


def _reduce(t: Tensor) -> Tensor:
    """``(E, 10, F)`` per row to the three filter groups."""
    return torch.stack([t[:, 0], t[:, 1:4].sum(1), t[:, 4:10].sum(1)], 1)


def _gather_sum(a: Tensor, x: Tensor, recv: Tensor, send: Tensor, n: int) -> Tensor:
    out = x.new_zeros(n, 10, x.shape[-1])
    return out.index_add_(0, recv, _expand(a) * x.index_select(0, send))


class _M(torch.autograd.Function):
    """Message sum onto the receivers."""

    @staticmethod
    @_records_mode
    def forward(ctx, a: Tensor, x: Tensor, plan: TensorPlan):
        ctx.save_for_backward(a, x)
        ctx.plan = plan
        if _kernels(a):
            return _ext.ops().tn_gather(plan.dst_ptr, plan.dst_order, plan.src, a.contiguous(), x.contiguous())
        return _gather_sum(a, x, plan.dst, plan.src, plan.n)

    @staticmethod
    @_keeps_mode
    def backward(ctx, g: Tensor):
        a, x = ctx.saved_tensors
        plan = ctx.plan
        da = _D.apply(g, x, plan) if ctx.needs_input_grad[0] else None
        dx = _MT.apply(a, g, plan) if ctx.needs_input_grad[1] else None
        return da, dx, None


class _MT(torch.autograd.Function):
    """Adjoint sum onto the senders: ``out[j] = sum_{j -> i} a (.) y[i]``."""

    @staticmethod
    @_records_mode
    def forward(ctx, a: Tensor, y: Tensor, plan: TensorPlan):
        ctx.save_for_backward(a, y)
        ctx.plan = plan
        if _kernels(a):
            return _ext.ops().tn_gather(plan.src_ptr, plan.src_order, plan.dst, a.contiguous(), y.contiguous())
        return _gather_sum(a, y, plan.src, plan.dst, plan.n)

    @staticmethod
    @_keeps_mode
    def backward(ctx, k: Tensor):
        a, y = ctx.saved_tensors
        plan = ctx.plan
        da = _D.apply(y, k, plan) if ctx.needs_input_grad[0] else None
        dy = _M.apply(a, k, plan) if ctx.needs_input_grad[1] else None
        return da, dy, None


class _D(torch.autograd.Function):
    """Per-pair group sums ``out[p, g] = sum_{c in g} y[dst, c] x[src, c]``."""

    @staticmethod
    @_records_mode
    def forward(ctx, y: Tensor, x: Tensor, plan: TensorPlan):
        ctx.save_for_backward(y, x)
        ctx.plan = plan
        if _kernels(y):
            return _ext.ops().tn_edge_dot(plan.dst, plan.src, y.contiguous(), x.contiguous())
        return _reduce(y.index_select(0, plan.dst) * x.index_select(0, plan.src))

    @staticmethod
    @_keeps_mode
    def backward(ctx, h: Tensor):
        y, x = ctx.saved_tensors
        plan = ctx.plan
        dy = _M.apply(h, x, plan) if ctx.needs_input_grad[0] else None
        dx = _MT.apply(h, y, plan) if ctx.needs_input_grad[1] else None
        return dy, dx, None


class _Em(torch.autograd.Function):
    """Embedding sum onto the receivers: ``out[i, c] = sum_{p -> i} a[p, g(c)] geo[p, c]``."""

    @staticmethod
    @_records_mode
    def forward(ctx, a: Tensor, geo: Tensor, plan: TensorPlan):
        ctx.save_for_backward(a, geo)
        ctx.plan = plan
        if _kernels(a):
            return _ext.ops().tn_embed(plan.dst_ptr, plan.dst_order, a.contiguous(), geo.contiguous())
        out = a.new_zeros(plan.n, 10, a.shape[-1])
        return out.index_add_(0, plan.dst, _expand(a) * geo.unsqueeze(-1))

    @staticmethod
    @_keeps_mode
    def backward(ctx, g: Tensor):
        a, geo = ctx.saved_tensors
        plan = ctx.plan
        da = _Ea.apply(g, geo, plan) if ctx.needs_input_grad[0] else None
        dgeo = _Eg.apply(a, g, plan) if ctx.needs_input_grad[1] else None
        return da, dgeo, None


class _Ea(torch.autograd.Function):
    """``out[p, g] = sum_{c in g} y[dst, c] geo[p, c]`` (the adjoint of the embedding in ``a``)."""

    @staticmethod
    @_records_mode
    def forward(ctx, y: Tensor, geo: Tensor, plan: TensorPlan):
        ctx.save_for_backward(y, geo)
        ctx.plan = plan
        if _kernels(y):
            return _ext.ops().tn_embed_da(plan.dst, y.contiguous(), geo.contiguous())
        return _reduce(y.index_select(0, plan.dst) * geo.unsqueeze(-1))

    @staticmethod
    @_keeps_mode
    def backward(ctx, h: Tensor):
        y, geo = ctx.saved_tensors
        plan = ctx.plan
        dy = _Em.apply(h, geo, plan) if ctx.needs_input_grad[0] else None
        dgeo = _Eg.apply(h, y, plan) if ctx.needs_input_grad[1] else None
        return dy, dgeo, None


class _Eg(torch.autograd.Function):
    """``out[p, c] = sum_f a[p, g(c), f] y[dst, c, f]`` (the adjoint of the embedding in ``geo``)."""

    @staticmethod
    @_records_mode
    def forward(ctx, a: Tensor, y: Tensor, plan: TensorPlan):
        ctx.save_for_backward(a, y)
        ctx.plan = plan
        if _kernels(a):
            return _ext.ops().tn_embed_dg(plan.dst, a.contiguous(), y.contiguous())
        return (_expand(a) * y.index_select(0, plan.dst)).sum(-1)

    @staticmethod
    @_keeps_mode
    def backward(ctx, k: Tensor):
        a, y = ctx.saved_tensors
        plan = ctx.plan
        da = _Ea.apply(y, k, plan) if ctx.needs_input_grad[0] else None
        dy = _Em.apply(a, k, plan) if ctx.needs_input_grad[1] else None
        return da, dy, None


def embedding(a: Tensor, geo: Tensor, plan: TensorPlan) -> Tensor:
    """``Em(a, geo)``: pair parts ``a (E, 3, F)`` weighing the geometry rows ``geo (E, 10)``
    (:func:`geometry_rows`) -> compact rows ``(n, 10, F)``."""
    return _Em.apply(a, geo, plan)


def geometry_rows(u: Tensor) -> Tensor:
    """``[1, u_x, u_y, u_z, u_x u_x, u_x u_y, u_x u_z, u_y u_y, u_y u_z, u_z u_z]`` per pair."""
    x, y, z = u.unbind(-1)
    return torch.stack([torch.ones_like(x), x, y, z, x * x, x * y, x * z, y * y, y * z, z * z], -1)


def messages(a: Tensor, x: Tensor, plan: TensorPlan) -> Tensor:
    """``M(a, x)``: filters ``a (E, 3, F)``, compact features ``x (n, 10, F)`` -> ``(n, 10, F)``."""
    return _M.apply(a, x, plan)


def to_compact(scalar: Tensor, vector: Tensor, sym: Tensor) -> Tensor:
    """``(n, F)``, ``(n, 3, F)``, full symmetric ``(n, 3, 3, F)`` -> compact rows ``(n, 10, F)``."""
    s6 = torch.stack([sym[:, 0, 0], sym[:, 0, 1], sym[:, 0, 2], sym[:, 1, 1], sym[:, 1, 2], sym[:, 2, 2]], 1)
    return torch.cat([scalar.unsqueeze(1), vector, s6], 1)


def sym_from_compact(s6: Tensor) -> Tensor:
    """Six distinct entries ``(n, 6, F)`` -> the full symmetric matrices ``(n, 3, 3, F)``."""
    xx, xy, xz, yy, yz, zz = s6.unbind(1)
    return torch.stack([xx, xy, xz, xy, yy, yz, xz, yz, zz], 1).reshape(s6.shape[0], 3, 3, s6.shape[2])


class _MM3(torch.autograd.Function):
    """``C = op(A) op(B)`` per atom and channel on ``(n, 3, 3, F)`` tensors (``op`` a transpose when
    its flag is set); the backward products are of the same kind, so any order differentiates."""

    @staticmethod
    @_records_mode
    def forward(ctx, A: Tensor, B: Tensor, ta: bool, tb: bool):
        ctx.save_for_backward(A, B)
        ctx.t = (ta, tb)
        if _kernels(A) and A.dtype == B.dtype:
            return _ext.ops().tn_mm3(A.contiguous(), B.contiguous(), bool(ta), bool(tb))
        a = A.transpose(1, 2) if ta else A
        b = B.transpose(1, 2) if tb else B
        return torch.einsum("nikf,nkjf->nijf", a, b)

    @staticmethod
    @_keeps_mode
    def backward(ctx, g: Tensor):
        A, B = ctx.saved_tensors
        ta, tb = ctx.t
        dA = dB = None
        if ctx.needs_input_grad[0]:
            dA = _MM3.apply(g, B, False, not tb) if not ta else _MM3.apply(B, g, tb, True)
        if ctx.needs_input_grad[1]:
            dB = _MM3.apply(A, g, not ta, False) if not tb else _MM3.apply(g, A, True, ta)
        return dA, dB, None, None


def matmul3(A: Tensor, B: Tensor, ta: bool = False, tb: bool = False) -> Tensor:
    """Per atom and channel 3x3 matrix products of ``(n, 3, 3, F)`` tensors."""
    return _MM3.apply(A, B, ta, tb)


class _PLin(torch.autograd.Function):
    """``[out1; out2] = M [in1; in2]`` per atom and channel (rows of ``(n, K, F)`` tensors, ``M``
    a constant ``(O, K)`` float64 matrix; ``out2`` only when ``O1 < O``, ``in2`` optional). Linear,
    so its backward is the same map with ``M^T`` and every order differentiates."""

    @staticmethod
    @_records_mode
    def forward(ctx, in1: Tensor, in2, M: Tensor, MT: Tensor, O1: int):
        ctx.K1 = in1.shape[1]
        ctx.O1 = O1
        ctx.two_in = in2 is not None
        ctx.mats = (M, MT)
        if _kernels(in1):
            o1, o2 = _ext.ops().tn_plin(in1.contiguous(), None if in2 is None else in2.contiguous(),
                                        M.to(in1.device), int(O1))
        else:
            x = in1 if in2 is None else torch.cat([in1, in2], 1)
            out = torch.einsum("ok,nkf->nof", M.to(x.dtype), x)
            o1, o2 = out[:, :O1].contiguous(), out[:, O1:].contiguous()
        if O1 == M.shape[0]:
            return o1
        return o1, o2

    @staticmethod
    @_keeps_mode
    def backward(ctx, *gs):
        M, MT = ctx.mats
        g1 = gs[0]
        g2 = gs[1] if len(gs) > 1 else None
        res = _PLin.apply(g1, g2, MT, M, ctx.K1)
        if ctx.two_in:
            d1, d2 = res
        else:
            d1, d2 = res, None
        return d1, d2, None, None, None


class LinearMap:
    """A constant per-atom, per-channel linear map of component rows (kernel ``tn_plin``)."""

    def __init__(self, M: Tensor, O1: Optional[int] = None):
        self.M = M.to(torch.float64).contiguous()
        self.MT = self.M.t().contiguous()
        self.O1 = int(M.shape[0] if O1 is None else O1)
        self._dev = {}

    def _on(self, dev):
        key = str(dev)
        if key not in self._dev:
            self._dev[key] = (self.M.to(dev), self.MT.to(dev))
        return self._dev[key]

    def __call__(self, in1: Tensor, in2: Optional[Tensor] = None):
        M, MT = self._on(in1.device)
        return _PLin.apply(in1, in2, M, MT, self.O1)


def _trace3(t: Tensor) -> Tensor:
    return (t[:, 0, 0] + t[:, 1, 1] + t[:, 2, 2]) / 3.0


def _matrix_of(fn, k_in: int) -> Tensor:
    """The matrix of a linear map of component rows, read off from the basis vectors."""
    eye = torch.eye(k_in, dtype=torch.float64)
    cols = [fn(eye[r].view(1, k_in, 1)).reshape(-1) for r in range(k_in)]
    return torch.stack(cols, 1)


def _parts(T: Tensor):
    """Scalar, skew and traceless symmetric parts of ``(1, 3, 3, 1)`` matrices."""
    skew = 0.5 * (T - T.transpose(1, 2))
    s = _trace3(T)
    sym = 0.5 * (T + T.transpose(1, 2)) - s[:, None, None] * torch.eye(3, dtype=T.dtype)[None, :, :, None]
    return s, skew, sym


def _compose(s: Tensor, skew: Tensor, sym: Tensor) -> Tensor:
    return s[:, None, None] * torch.eye(3, dtype=skew.dtype)[None, :, :, None] + skew + sym


def _axial(t: Tensor) -> Tensor:
    return 0.5 * torch.stack([t[:, 2, 1] - t[:, 1, 2], t[:, 0, 2] - t[:, 2, 0], t[:, 1, 0] - t[:, 0, 1]], 1)


def _three_parts(x: Tensor):
    """``(1, 27, 1)`` rows ``k * 3 + j`` (matrix entry ``k``, product ``j``) -> the scalar part of
    product 0, the skew part of product 1 and the traceless symmetric part of product 2."""
    G = x.view(1, 9, 3, 1)
    s = _parts(G[:, :, 0].reshape(1, 3, 3, 1))[0]
    skew = _parts(G[:, :, 1].reshape(1, 3, 3, 1))[1]
    sym = _parts(G[:, :, 2].reshape(1, 3, 3, 1))[2]
    return s, skew, sym


def _y_and_compact(x: Tensor) -> Tensor:
    s, skew, sym = _three_parts(x)
    Y = _compose(s, skew, sym).reshape(1, 9, 1)
    c = torch.cat([s.unsqueeze(1), _axial(skew), torch.stack([sym[:, 0, 0], sym[:, 0, 1], sym[:, 0, 2],
                                                              sym[:, 1, 1], sym[:, 1, 2], sym[:, 2, 2]], 1)], 1)
    return torch.cat([Y, c], 1)


def _full_from_compact(x: Tensor) -> Tensor:
    m = x.view(1, 10, 1)
    v = m[:, 1:4]
    z = torch.zeros_like(v[:, 0])
    skew = torch.stack([z, -v[:, 2], v[:, 1], v[:, 2], z, -v[:, 0], -v[:, 1], v[:, 0], z], 1).reshape(1, 3, 3, 1)
    return _compose(m[:, 0], skew, sym_from_compact(m[:, 4:10])).reshape(1, 9, 1)


#: (Y | compact rows) of the three channel products of a normalised tensor (27 -> 9 + 10)
Y_AND_COMPACT = LinearMap(_matrix_of(_y_and_compact, 27), O1=9)
#: full 3x3 rows of compact rows (10 -> 9)
FULL_FROM_COMPACT = LinearMap(_matrix_of(_full_from_compact, 10))
#: scalar / skew / traceless symmetric parts of three products, recomposed (27 -> 9)
RECOMPOSE = LinearMap(_matrix_of(lambda x: _compose(*_three_parts(x)).reshape(1, 9, 1), 27))


def _embedding_full(x: Tensor) -> Tensor:
    m = x.view(1, 10, 1)
    full = _full_from_compact(x).view(1, 3, 3, 1)
    sym = sym_from_compact(m[:, 4:10])
    return (full - (_trace3(sym))[:, None, None] * torch.eye(3, dtype=x.dtype)[None, :, :, None]).reshape(1, 9, 1)


#: the embedding's tensors from its summed rows: scalar, skew of the vector, traceless symmetric (10 -> 9)
EMBEDDING_FULL = LinearMap(_matrix_of(_embedding_full, 10))
