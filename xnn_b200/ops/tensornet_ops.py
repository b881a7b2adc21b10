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
functions run their PyTorch formulas.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from .. import _ext

GROUP = (0, 1, 1, 1, 2, 2, 2, 2, 2, 2)


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
    if not t.is_cuda or t.dtype not in (torch.float32, torch.float64) or t.shape[-1] > 128:
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
    def forward(ctx, a: Tensor, x: Tensor, plan: TensorPlan):
        ctx.save_for_backward(a, x)
        ctx.plan = plan
        if _kernels(a):
            return _ext.ops().tn_gather(plan.dst_ptr, plan.dst_order, plan.src, a.contiguous(), x.contiguous())
        return _gather_sum(a, x, plan.dst, plan.src, plan.n)

    @staticmethod
    def backward(ctx, g: Tensor):
        a, x = ctx.saved_tensors
        plan = ctx.plan
        da = _D.apply(g, x, plan) if ctx.needs_input_grad[0] else None
        dx = _MT.apply(a, g, plan) if ctx.needs_input_grad[1] else None
        return da, dx, None


class _MT(torch.autograd.Function):
    """Adjoint sum onto the senders: ``out[j] = sum_{j -> i} a (.) y[i]``."""

    @staticmethod
    def forward(ctx, a: Tensor, y: Tensor, plan: TensorPlan):
        ctx.save_for_backward(a, y)
        ctx.plan = plan
        if _kernels(a):
            return _ext.ops().tn_gather(plan.src_ptr, plan.src_order, plan.dst, a.contiguous(), y.contiguous())
        return _gather_sum(a, y, plan.src, plan.dst, plan.n)

    @staticmethod
    def backward(ctx, k: Tensor):
        a, y = ctx.saved_tensors
        plan = ctx.plan
        da = _D.apply(y, k, plan) if ctx.needs_input_grad[0] else None
        dy = _M.apply(a, k, plan) if ctx.needs_input_grad[1] else None
        return da, dy, None


class _D(torch.autograd.Function):
    """Per-pair group sums ``out[p, g] = sum_{c in g} y[dst, c] x[src, c]``."""

    @staticmethod
    def forward(ctx, y: Tensor, x: Tensor, plan: TensorPlan):
        ctx.save_for_backward(y, x)
        ctx.plan = plan
        if _kernels(y):
            return _ext.ops().tn_edge_dot(plan.dst, plan.src, y.contiguous(), x.contiguous())
        return _reduce(y.index_select(0, plan.dst) * x.index_select(0, plan.src))

    @staticmethod
    def backward(ctx, h: Tensor):
        y, x = ctx.saved_tensors
        plan = ctx.plan
        dy = _M.apply(h, x, plan) if ctx.needs_input_grad[0] else None
        dx = _MT.apply(h, y, plan) if ctx.needs_input_grad[1] else None
        return dy, dx, None


class _Em(torch.autograd.Function):
    """Embedding sum onto the receivers: ``out[i, c] = sum_{p -> i} a[p, g(c)] geo[p, c]``."""

    @staticmethod
    def forward(ctx, a: Tensor, geo: Tensor, plan: TensorPlan):
        ctx.save_for_backward(a, geo)
        ctx.plan = plan
        if _kernels(a):
            return _ext.ops().tn_embed(plan.dst_ptr, plan.dst_order, a.contiguous(), geo.contiguous())
        out = a.new_zeros(plan.n, 10, a.shape[-1])
        return out.index_add_(0, plan.dst, _expand(a) * geo.unsqueeze(-1))

    @staticmethod
    def backward(ctx, g: Tensor):
        a, geo = ctx.saved_tensors
        plan = ctx.plan
        da = _Ea.apply(g, geo, plan) if ctx.needs_input_grad[0] else None
        dgeo = _Eg.apply(a, g, plan) if ctx.needs_input_grad[1] else None
        return da, dgeo, None


class _Ea(torch.autograd.Function):
    """``out[p, g] = sum_{c in g} y[dst, c] geo[p, c]`` (the adjoint of the embedding in ``a``)."""

    @staticmethod
    def forward(ctx, y: Tensor, geo: Tensor, plan: TensorPlan):
        ctx.save_for_backward(y, geo)
        ctx.plan = plan
        if _kernels(y):
            return _ext.ops().tn_embed_da(plan.dst, y.contiguous(), geo.contiguous())
        return _reduce(y.index_select(0, plan.dst) * geo.unsqueeze(-1))

    @staticmethod
    def backward(ctx, h: Tensor):
        y, geo = ctx.saved_tensors
        plan = ctx.plan
        dy = _Em.apply(h, geo, plan) if ctx.needs_input_grad[0] else None
        dgeo = _Eg.apply(h, y, plan) if ctx.needs_input_grad[1] else None
        return dy, dgeo, None


class _Eg(torch.autograd.Function):
    """``out[p, c] = sum_f a[p, g(c), f] y[dst, c, f]`` (the adjoint of the embedding in ``geo``)."""

    @staticmethod
    def forward(ctx, a: Tensor, y: Tensor, plan: TensorPlan):
        ctx.save_for_backward(a, y)
        ctx.plan = plan
        if _kernels(a):
            return _ext.ops().tn_embed_dg(plan.dst, a.contiguous(), y.contiguous())
        return (_expand(a) * y.index_select(0, plan.dst)).sum(-1)

    @staticmethod
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
    def forward(ctx, A: Tensor, B: Tensor, ta: bool, tb: bool):
        ctx.save_for_backward(A, B)
        ctx.t = (ta, tb)
        if _kernels(A) and A.dtype == B.dtype:
            return _ext.ops().tn_mm3(A.contiguous(), B.contiguous(), bool(ta), bool(tb))
        a = A.transpose(1, 2) if ta else A
        b = B.transpose(1, 2) if tb else B
        return torch.einsum("nikf,nkjf->nijf", a, b)

    @staticmethod
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
