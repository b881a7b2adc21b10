"""Fused ops of the equivariant message pass, differentiable to second order.

On CUDA every op is a kernel of ``xnn_b200._C`` wrapped in an autograd Function whose
backward is itself a Function of kernels (and whose second backward is once more
kernels), so the double backward of a force loss runs entirely on the fused kernels:

* :func:`edge_geometry` -- spherical harmonics and enveloped Bessel basis of the edge
  vectors; VJP and JVP kernels (exact, forward-mode dual numbers).
* :func:`conv` -- the gather / uvu product / scatter-sum message pass as the derivative
  of one 4-linear form (see ``csrc/conv.cu``); all of its derivatives are the same four
  contractions.
* :func:`symmetric_contraction` -- MACE's per-element polynomial of the coupled
  features (``csrc/symcon.cu``).

On the CPU the same functions evaluate the same mathematics with PyTorch operations
(autograd then provides the derivatives), which is what the tests compare against.
"""
from __future__ import annotations

import functools
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
from torch import Tensor
from torch.autograd import Function
from torch.autograd.function import once_differentiable

from .. import _ext
from .modes import MODES


def _C():
    return _ext.ops()


def _use_kernels(t: Tensor) -> bool:
    if not t.is_cuda:
        return False
    if not _ext.cuda_available():
        raise RuntimeError("xnn_b200: fused CUDA path requested but the native extension is "
                           f"not available ({_ext.error()}); build it with xnn_b200.build.build()")
    return True


# --------------------------------------------------------------------------- edge plan
@dataclass
class EdgePlan:
    """CSR views of one edge list: edges grouped by receiver and by sender."""

    n_nodes: int
    n_edges: int
    src32: Tensor
    dst32: Tensor
    src: Tensor
    dst: Tensor
    dst_ptr: Tensor
    dst_perm: Optional[Tensor]
    src_ptr: Optional[Tensor]
    src_perm: Optional[Tensor]
    #: number of sender rows when senders and receivers differ (an edge chunk); -1: ``n_nodes``
    n_src: int = -1

    @property
    def n_senders(self) -> int:
        return self.n_src if self.n_src >= 0 else self.n_nodes

    @staticmethod
    def from_packed(edge_index: Tensor, n_nodes: int, packed: Tensor) -> "EdgePlan":
        """The plan of receiver-sorted edges from ``[dst_ptr | src_ptr | src_perm]`` computed on
        the host (no sort on the device)."""
        src, dst = edge_index[0], edge_index[1]
        E = int(src.shape[0])
        n1 = n_nodes + 1
        return EdgePlan(n_nodes, E, src.to(torch.int32), dst.to(torch.int32), src, dst, packed[:n1],
                        None, packed[n1:2 * n1], packed[2 * n1:2 * n1 + E])

    @staticmethod
    def build(edge_index: Tensor, n_nodes: int, assume_dst_sorted: Optional[bool] = None,
              n_src: Optional[int] = None, senders: bool = True) -> "EdgePlan":
        src, dst = edge_index[0], edge_index[1]
        E = int(src.shape[0])
        dev = src.device
        # counts by index_add (no host synchronisation: capturable in a CUDA graph)
        one = torch.ones(E, dtype=torch.int64, device=dev)
        counts = torch.zeros(n_nodes, dtype=torch.int64, device=dev).index_add_(0, dst, one)
        dst_ptr = torch.zeros(n_nodes + 1, dtype=torch.int64, device=dev)
        dst_ptr[1:] = torch.cumsum(counts, 0)
        if assume_dst_sorted is None:
            assume_dst_sorted = bool((dst[1:] >= dst[:-1]).all()) if E > 1 else True
        dst_perm = None if assume_dst_sorted else torch.argsort(dst, stable=True)
        ns = n_nodes if n_src is None else int(n_src)
        plan = EdgePlan(n_nodes, E, src.to(torch.int32).contiguous(), dst.to(torch.int32).contiguous(),
                        src, dst, dst_ptr, dst_perm, None, None, -1 if n_src is None else ns)
        return plan.with_senders() if senders else plan

    def with_senders(self) -> "EdgePlan":
        """The plan with its sender ordering (``src_ptr``, ``src_perm``), formed on first use."""
        if self.src_ptr is None:
            ns, dev = self.n_senders, self.src.device
            one = torch.ones(self.n_edges, dtype=torch.int64, device=dev)
            scounts = torch.zeros(ns, dtype=torch.int64, device=dev).index_add_(0, self.src, one)
            self.src_ptr = torch.zeros(ns + 1, dtype=torch.int64, device=dev)
            self.src_ptr[1:] = torch.cumsum(scounts, 0)
            self.src_perm = torch.argsort(self.src, stable=True)
        return self


# --------------------------------------------------------------------------- edge geometry
def edge_features_torch(vec: Tensor, lmax: int, freqs: Tensor, norm: float, rc: float, p: int
                        ) -> Tuple[Tensor, Tensor]:
    """Reference formulas of :func:`edge_geometry` in PyTorch operations."""
    from ..o3 import spherical_harmonics
    Y = spherical_harmonics(list(range(lmax + 1)), vec, normalize=True, normalization="component")
    r = torch.linalg.norm(vec, dim=-1)
    rcl = r.clamp(min=1e-8)[:, None]
    bessel = norm * torch.sin(freqs * rcl / rc) / rcl
    x = r / rc
    poly = ((-(p * (p + 1) / 2.0)) * x + p * (p + 2.0)) * x - (p + 1) * (p + 2) / 2.0
    env = (1.0 + poly * x ** p) * (r < rc)
    return Y, bessel * env[:, None]


class _EdgeGeometry(Function):
    @staticmethod
    def forward(ctx, vec, freqs, cfg):
        lmax, norm, rc, p = cfg
        Y, R = _C().edge_geometry_fwd(vec.contiguous(), lmax, freqs.contiguous(), norm, rc, p)
        ctx.save_for_backward(vec, freqs)
        ctx.cfg = cfg
        return Y, R

    @staticmethod
    def backward(ctx, gY, gR):
        vec, freqs = ctx.saved_tensors
        if not ctx.needs_input_grad[0]:
            return None, None, None
        return _EdgeGeometryVJP.apply(vec, gY, gR, freqs, ctx.cfg), None, None


class _EdgeGeometryVJP(Function):
    @staticmethod
    def forward(ctx, vec, gY, gR, freqs, cfg):
        lmax, norm, rc, p = cfg
        gY_ = gY.contiguous() if gY is not None else None
        gR_ = gR.contiguous() if gR is not None else None
        gvec = _C().edge_geometry_bwd(vec.contiguous(), lmax, freqs, norm, rc, p, gY_, gR_)
        ctx.save_for_backward(vec, gY, gR, freqs)
        ctx.cfg = cfg
        ctx.set_materialize_grads(False)
        return gvec

    @staticmethod
    @once_differentiable
    def backward(ctx, u):
        vec, gY, gR, freqs = ctx.saved_tensors
        lmax, norm, rc, p = ctx.cfg
        if u is None:
            return None, None, None, None, None
        need_Y, need_R = ctx.needs_input_grad[1], ctx.needs_input_grad[2]
        dY = dR = None
        if need_Y or need_R:
            dY, dR = _C().edge_geometry_jvp(vec.contiguous(), lmax, freqs, norm, rc, p, u.contiguous(),
                                            bool(need_Y), bool(need_R))
            dY = dY if need_Y else None
            dR = dR if need_R else None
        dvec = None
        if ctx.needs_input_grad[0] and not MODES.params_only:
            with torch.enable_grad():
                v = vec.detach().requires_grad_(True)
                Yt, Rt = edge_features_torch(v, lmax, freqs, norm, rc, p)
                s = 0
                if gY is not None:
                    s = s + (Yt * gY).sum()
                if gR is not None:
                    s = s + (Rt * gR).sum()
                (g,) = torch.autograd.grad(s, v, create_graph=True)
                (dvec,) = torch.autograd.grad((g * u).sum(), v)
        return dvec, dY, dR, None, None


def edge_geometry(vec: Tensor, lmax: int, freqs: Tensor, norm: float, rc: float, p: int
                  ) -> Tuple[Tensor, Tensor]:
    """``(Y (E, (lmax+1)^2), radial (E, n_rbf))`` of the edge vectors (see module notes)."""
    if _use_kernels(vec) and lmax <= 3 and freqs.numel() <= 16 and not freqs.requires_grad:
        return _EdgeGeometry.apply(vec, freqs.to(vec.dtype), (int(lmax), float(norm), float(rc), int(p)))
    return edge_features_torch(vec, lmax, freqs, norm, rc, p)


# --------------------------------------------------------------------------- convolution
def _gather_torch(plan: EdgePlan, P: int, terms):
    D = P * P
    out = None
    lidx = torch.repeat_interleave(torch.arange(P), torch.tensor([2 * l + 1 for l in range(P)]))
    for x, R, Y in terms:
        xs = x.index_select(0, plan.src)                          # (E, C)
        msg = (R[:, lidx.to(R.device), :] * xs[:, None, :]) * Y[:, :, None]   # (E, D, C)
        part = torch.zeros(D, plan.n_nodes, x.shape[1], dtype=x.dtype, device=x.device)
        part = part.index_add(1, plan.dst, msg.transpose(0, 1))
        out = part if out is None else out + part
    return out


def conv_torch(x: Tensor, R: Tensor, Y: Tensor, plan: EdgePlan) -> Tensor:
    """The message pass in PyTorch operations (``A (D, N, C)``)."""
    P = R.shape[1]
    return _gather_torch(plan, P, [(x, R, Y)])


class _Conv(Function):
    @staticmethod
    def forward(ctx, x, R, Y, plan):
        N, C = plan.n_nodes, x.shape[1]
        P = R.shape[1]
        A = _C().conv_gather(N, C, P, plan.dst_ptr, plan.src32, plan.dst_perm, [x.contiguous()],
                             [R.contiguous()], [Y.contiguous()])
        ctx.save_for_backward(x, R, Y)
        ctx.plan = plan
        return A

    @staticmethod
    def backward(ctx, G):
        x, R, Y = ctx.saved_tensors
        nx, nR, nY = ctx.needs_input_grad[:3]
        if MODES.params_only:
            nY = False
        gx, gR, gY = _ConvVJP.apply(G, x, R, Y, ctx.plan, (bool(nx), bool(nR), bool(nY)))
        return gx, gR, gY, None


class _ConvVJP(Function):
    @staticmethod
    def forward(ctx, G, x, R, Y, plan, need):
        # T1[e, l, c] = sum_m G[lm, d, c] Y[e, lm]: gR = x[s] * T1, gx = sum_{e out of s} sum_l R * T1;
        # kept for the second derivative
        nx, nR, nY = need
        N, C, P = plan.n_nodes, x.shape[1], R.shape[1]
        G = G.contiguous()
        K = _C()
        gR, gY, T1, _, _ = K.conv_edge(N, C, P, plan.n_edges, plan.dst_ptr, plan.src32, plan.dst_perm, G,
                                    [Y], [x if nR else None], [True], bool(nR),
                                    [x] if nY else [], [R] if nY else [])
        gx = K.conv_scatter(plan.n_senders, C, P, plan.with_senders().src_ptr, plan.src_perm, [R], [T1]) if nx else None
        ctx.save_for_backward(G, x, R, Y, T1)
        ctx.plan = plan
        ctx.set_materialize_grads(False)
        return gx, (gR if nR else None), (gY if nY else None)

    @staticmethod
    @once_differentiable
    def backward(ctx, ux, uR, uY):
        G, x, R, Y, T1 = ctx.saved_tensors
        plan = ctx.plan
        N, C, P = plan.n_nodes, x.shape[1], R.shape[1]
        K = _C()
        nG, nx, nR, nY = ctx.needs_input_grad[:4]
        if MODES.params_only:
            nY = False
        ux = ux.contiguous() if ux is not None else None
        uR = uR.contiguous() if uR is not None else None
        uY = uY.contiguous() if uY is not None else None
        cG = cx = cR = cY = None
        if nG:
            xs, Rs, Ys = [], [], []
            for tx, tR, tY in ((ux, R, Y), (x, uR, Y), (x, R, uY)):
                if tx is not None and tR is not None and tY is not None:
                    xs.append(tx); Rs.append(tR); Ys.append(tY)
            if xs:
                cG = K.conv_gather(N, C, P, plan.dst_ptr, plan.src32, plan.dst_perm, xs, Rs, Ys)
        # edge terms: (Y, ux) gives ux*T1 to cot_R; (uY, x) gives x*T2 to cot_R and T2 for cot_x
        Ys, xs, wT = [], [], []
        if nR and ux is not None:
            Ys.append(Y); xs.append(ux); wT.append(False)
        if uY is not None and (nR or nx):
            Ys.append(uY); xs.append(x if nR else None); wT.append(bool(nx))
        xY, RY = [], []
        if nY:
            for tx, tR in ((ux, R), (x, uR)):
                if tx is not None and tR is not None:
                    xY.append(tx); RY.append(tR)
        T2 = None
        if Ys or xY:
            a, b, t0, t1, _ = K.conv_edge(N, C, P, plan.n_edges, plan.dst_ptr, plan.src32, plan.dst_perm, G,
                                       Ys, xs, wT, bool(nR) and any(v is not None for v in xs), xY, RY)
            cR = a if (nR and any(v is not None for v in xs)) else None
            cY = b if xY else None
            if uY is not None and nx:
                T2 = t1 if len(Ys) == 2 else t0
        if nx:
            As, Bs = [], []
            if uR is not None:
                As.append(uR); Bs.append(T1)
            if T2 is not None:
                As.append(R); Bs.append(T2)
            if As:
                cx = K.conv_scatter(plan.n_senders, C, P, plan.with_senders().src_ptr, plan.src_perm, As, Bs)
        return cG, cx, cR, cY, None, None


def conv(x: Tensor, R: Tensor, Y: Tensor, plan: EdgePlan) -> Tensor:
    """``A[lm, d, c] = sum_{e: s->d} R[e, l, c] x[s, c] Y[e, lm]`` for scalar node features.

    ``x (N, C)``, ``R (E, P, C)``, ``Y (E, P*P)``; returns ``A (P*P, N, C)``.
    """
    if _use_kernels(x):
        return _Conv.apply(x, R, Y, plan)
    return conv_torch(x, R, Y, plan)


# --------------------------------------------------------------------------- symmetric contraction
@functools.lru_cache(maxsize=None)
def _monomials(lmax: int, corr: int):
    from ..csrc.gen_symcon import monomials
    orders = monomials(lmax, corr)
    K = sum(k for _, k, _ in orders)
    D = (lmax + 1) ** 2
    ks, cs, idx = [], [], []
    for _, _, lst in orders:
        for k, ix, c in lst:
            ks.append(k)
            cs.append(c)
            idx.append(list(ix) + [D] * (3 - len(ix)))
    return K, torch.tensor(ks), torch.tensor(cs, dtype=torch.float64), torch.tensor(idx)


def num_invariants(lmax: int, corr: int) -> int:
    return _monomials(lmax, corr)[0]


def invariants_torch(A: Tensor, lmax: int, corr: int) -> Tensor:
    """``I (K, N, C)`` of the coupled components ``A (D, N, C)``."""
    K, ks, cs, idx = _monomials(lmax, corr)
    ones = torch.ones_like(A[:1])
    Ap = torch.cat([A, ones], 0)                      # index D is the constant 1
    idx = idx.to(A.device)
    prod = Ap[idx[:, 0]] * Ap[idx[:, 1]] * Ap[idx[:, 2]]          # (T, N, C)
    prod = prod * cs.to(A.device, A.dtype)[:, None, None]
    out = torch.zeros((K,) + tuple(A.shape[1:]), dtype=A.dtype, device=A.device)
    return out.index_add(0, ks.to(A.device), prod)


def symmetric_contraction_torch(A: Tensor, W: Tensor, z: Tensor, lmax: int, corr: int) -> Tensor:
    I = invariants_torch(A, lmax, corr)               # (K, N, C)
    Wa = W.index_select(0, z)                         # (N, K, C)
    return (Wa * I.transpose(0, 1)).sum(1)


class _Symcon(Function):
    @staticmethod
    def forward(ctx, A, W, z, cfg):
        lmax, corr = cfg
        out = _C().symcon_fwd(A.contiguous(), z, W.contiguous(), lmax, corr)
        ctx.save_for_backward(A, W, z)
        ctx.cfg = cfg
        return out

    @staticmethod
    def backward(ctx, g):
        A, W, z = ctx.saved_tensors
        need_A = bool(ctx.needs_input_grad[0])
        need_W = bool(ctx.needs_input_grad[1]) and not MODES.force_pass
        if not (need_A or need_W):
            return None, None, None, None
        gA, gW = _SymconVJP.apply(A, W, g, z, ctx.cfg, need_A, need_W)
        return gA, gW, None, None


class _SymconVJP(Function):
    @staticmethod
    def forward(ctx, A, W, g, z, cfg, need_A, need_W):
        lmax, corr = cfg
        g = g.contiguous()
        gA, gWa = _C().symcon_bwd(A.contiguous(), z, W.contiguous(), g, lmax, corr, need_A, need_W)
        gW = None
        if need_W:
            gW = torch.zeros_like(W).index_add_(0, z, gWa)
        ctx.save_for_backward(A, W, g, z)
        ctx.cfg = cfg
        ctx.set_materialize_grads(False)
        return (gA if need_A else None), gW

    @staticmethod
    @once_differentiable
    def backward(ctx, uA, uW):
        A, W, g, z = ctx.saved_tensors
        lmax, corr = ctx.cfg
        nA, nW, ng = ctx.needs_input_grad[:3]
        if uA is None and uW is None:
            return None, None, None, None, None, None, None
        uWa = uW.index_select(0, z).contiguous() if uW is not None else None
        cg, cA, cWa = _C().symcon_bwd2(A.contiguous(), z, W.contiguous(), g,
                                       uA.contiguous() if uA is not None else None, uWa, lmax, corr,
                                       bool(ng), bool(nA), bool(nW))
        cW = torch.zeros_like(W).index_add_(0, z, cWa) if nW else None
        return (cA if nA else None), cW, (cg if ng else None), None, None, None, None


def symmetric_contraction(A: Tensor, W: Tensor, z: Tensor, lmax: int, corr: int) -> Tensor:
    """``out[i, c] = sum_k W[z_i, k, c] I_k(A[:, i, c])`` with ``A (D, N, C)``, ``W (n_el, K, C)``."""
    if _use_kernels(A):
        return _Symcon.apply(A, W, z, (int(lmax), int(corr)))
    return symmetric_contraction_torch(A, W, z, lmax, corr)
