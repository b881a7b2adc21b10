"""Radial network + message pass for force evaluation on millions of edges, in bounded memory.

``A[lm, d, c] = sum_{e: s->d} R(r_e)[l, c] x[s, c] Y[e, lm]`` evaluated over receiver-contiguous
edge chunks; the per-edge tensors of the radial network (``R``, its tangent ``dR/dr`` and the
hidden activations, several kB per edge) exist for one chunk at a time and are never saved.
The backward recomputes ``R`` and ``dR/dr`` chunk by chunk (the forward-mode network of
:mod:`xnn_b200.ops.radial`) and forms, per chunk, the edge cotangents ``g_r = sum gR dR/dr`` and
``gY`` and each edge's term of the sender cotangent (an ``(E, C)`` row, summed per sender by a
second kernel), so no ``(E, P, C)`` tensor besides ``R`` and ``dR/dr`` is written. Saved state is ``x``, ``r`` and ``Y``: O(E) floats
instead of O(E * P * C).

First derivatives only (forces, stress, MD); parameter gradients are not formed, so training
uses the ordinary path. CUDA only.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
from torch import Tensor
from torch.autograd import Function
from torch.autograd.function import once_differentiable
from torch.nn import functional as F

from .. import _ext
from . import gemm
from .mace_ops import EdgePlan
from .radial import RadialSpec, _eff, _forward


def _primal(r: Tensor, We: List[Tensor], spec: RadialSpec) -> Tensor:
    """``R`` only (no tangent rows): basis, hidden SiLU layers (fused into the products'
    epilogue where the tensor-core kernel takes them), output layer."""
    E = r.shape[0]
    H = _ext.ops().radial_basis(r.contiguous(), spec.freqs.to(r.device), spec.norm, spec.rc, spec.p)[:E]
    for k in range(len(We) - 1):
        Hk = gemm.mm_act(H.contiguous(), We[k], 1, spec.consts[k])
        if Hk is None:
            Hk = F.silu(gemm.mm_raw(H.contiguous(), We[k]))
            if spec.consts[k] != 1.0:
                Hk = Hk * spec.consts[k]
        H = Hk
    return gemm.mm_raw(H.contiguous(), We[-1])


def _primal_tangent(r: Tensor, We: List[Tensor], spec: RadialSpec) -> Optional[Tuple[Tensor, Tensor]]:
    """``R`` and ``dR/dr``: the value and tangent columns side by side (``[h | h']``), each hidden
    layer one product with the block-diagonal weight and the coupled activation in its epilogue."""
    E = r.shape[0]
    B = _ext.ops().radial_basis(r.contiguous(), spec.freqs.to(r.device), spec.norm, spec.rc, spec.p)
    H = torch.cat([B[:E], B[E:]], 1)
    for k in range(len(We) - 1):
        Hk = gemm.mm_act(H, torch.block_diag(We[k], We[k]), 2, spec.consts[k])
        if Hk is None:
            return None
        H = Hk
    n = H.shape[1] // 2
    return gemm.mm_raw(H[:, :n], We[-1]), gemm.mm_raw(H[:, n:], We[-1])


Chunk = Tuple[Tuple[int, int], Tuple[int, int], EdgePlan]


class _LeanRadialConv(Function):
    @staticmethod
    def forward(ctx, x: Tensor, r: Tensor, Y: Tensor, chunks: Sequence[Chunk], spec: RadialSpec, P: int,
                plan: Optional[EdgePlan], *Ws: Tensor) -> Tensor:
        C = x.shape[1]
        N = chunks[-1][1][1]
        K = _ext.ops()
        We = _eff(Ws, spec)
        A = x.new_empty((P * P, N, C))
        xc = x.contiguous()
        for (e0, e1), (n0, n1), sub in chunks:
            R = _primal(r[e0:e1], We, spec).view(-1, P, C)
            A[:, n0:n1] = K.conv_gather(n1 - n0, C, P, sub.dst_ptr, sub.src32, None, [xc], [R],
                                        [Y[e0:e1].contiguous()])
        ctx.chunks, ctx.spec, ctx.P, ctx.plan = chunks, spec, P, plan
        ctx.save_for_backward(x, r, Y, *Ws)
        return A

    @staticmethod
    @once_differentiable
    def backward(ctx, G: Tensor):
        x, r, Y = ctx.saved_tensors[:3]
        Ws = ctx.saved_tensors[3:]
        P, spec = ctx.P, ctx.spec
        N_src, C = x.shape
        K = _ext.ops()
        We = _eff(Ws, spec)
        xc = x.contiguous()
        want_x = ctx.needs_input_grad[0]
        gx = None
        g_r = torch.empty_like(r) if ctx.needs_input_grad[1] else None
        gY = torch.empty_like(Y) if ctx.needs_input_grad[2] else None
        # the edges' sender terms of every chunk in one (E, C) buffer, summed per sender once over
        # the whole graph's sender ordering; per chunk when that buffer does not fit
        plan = ctx.plan
        E = r.shape[0]
        whole = want_x and plan is not None and 2 * E * C * x.element_size() < torch.cuda.mem_get_info(x.device)[0]
        gxe_all = x.new_empty((E, C)) if whole else None
        if want_x and not whole:
            gx = torch.zeros_like(xc)
        for (e0, e1), (n0, n1), sub in ctx.chunks:
            fused = _primal_tangent(r[e0:e1], We, spec)
            R, Rd = fused if fused is not None else _forward(r[e0:e1], We, spec)[:2]
            R, Rd = R.view(-1, P, C), Rd.view(-1, P, C)
            Gc = G[:, n0:n1].contiguous()
            Yc = Y[e0:e1].contiguous()
            # the force kernel contracts gR with dR/dr itself (g_r without the (E, P, C) gR tensor)
            # and writes each edge's (E, C) term of the sender cotangent, summed per sender after
            g_rc, gYc, gxe = K.conv_force(n1 - n0, C, P, e1 - e0, sub.dst_ptr, sub.src32, Gc, Yc, xc,
                                          R.contiguous(), Rd.contiguous(), gxe_all[e0:e1] if whole else None)
            if g_r is not None:
                g_r[e0:e1] = g_rc
            if gY is not None:
                gY[e0:e1] = gYc
            if want_x and not whole:
                sub = sub.with_senders()
                gx += K.conv_sender_sum(N_src, sub.src_ptr, sub.src_perm, gxe)
        if whole:
            plan = plan.with_senders()
            gx = K.conv_sender_sum(N_src, plan.src_ptr, plan.src_perm, gxe_all)
        return (gx, g_r, gY, None, None, None, None) + (None,) * len(Ws)


def lean_radial_conv(x: Tensor, r: Tensor, Y: Tensor, chunks: Sequence[Chunk], net, col_scale: Tensor,
                     freqs: Tensor, norm: float, rc: float, p: int, P: int,
                     plan: Optional[EdgePlan] = None) -> Tensor:
    """``A (P*P, N, C)`` of the MACE message pass with the radial network ``net`` (see module notes);
    ``plan``: the whole graph's edge plan (sender ordering of the chunks' edges taken together)."""
    spec = RadialSpec(net, col_scale, freqs, norm, rc, p)
    Ws = [layer.weight for layer in net]
    return _LeanRadialConv.apply(x, r, Y, chunks, spec, P, plan, *Ws)
