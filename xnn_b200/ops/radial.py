"""The per-edge radial network of MACE / NequIP, differentiated forward-mode along the edge length.

The network ``R(r) = MLP(rad(r))`` depends on the edge vector only through its length ``r``
(``rad`` is the enveloped Bessel basis). The forward pass therefore carries the tangent
``dR/dr`` next to ``R``: primal and tangent rows are stacked, so every layer is one matrix
product over ``2E`` rows, and the activation couples the halves
(``h = c f(a)``, ``h' = c f'(a) a'``). Consequences for a force-loss step:

* force pass: ``dE/dr = sum_j gR[e, j] dR/dr[e, j]`` -- no matrix product at all;
* parameter pass: the energy term is one reverse sweep over the primal rows; the force term is
  one reverse sweep of the stacked network with cotangent ``u_r gR`` on the tangent rows, whose
  activation derivative brings in ``f''``.

Weights are the e3nn-layout ``layer{k}.weight`` parameters; the per-layer normalisation
factors and constants are applied inside (``FullyConnectedNet.folded``), the per-column
scale of the last layer carries the tensor-product path coefficients.

On CUDA the stages are kernels of ``xnn_b200._C``: the stacked basis, the coupled activation and
its reverse (``csrc/radial_kernels.cu``), the row products and the weight-gradient reductions on
the tensor cores (``csrc/gemm_tc*.cu``, 3xTF32 for float32). On the CPU the same formulas run
as PyTorch operations.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
from torch import Tensor
from torch.autograd import Function
from torch.autograd.function import once_differentiable

from .. import _ext
from . import gemm
from .modes import MODES


# ------------------------------------------------------------------------------- stages
def _silu_d(a: Tensor):
    s = torch.sigmoid(a)
    f = a * s
    f1 = s * (1.0 + a * (1.0 - s))
    f2 = s * (1.0 - s) * (2.0 + a * (1.0 - 2.0 * s))
    return f, f1, f2


def bessel_envelope(r: Tensor, freqs: Tensor, norm: float, rc: float, p: int) -> Tuple[Tensor, Tensor]:
    """``rad (E, n)`` and ``d rad / dr`` of ``norm sin(f r / rc) / r * env(r / rc)``."""
    rcl = r.clamp(min=1e-8)[:, None]
    w = freqs / rc
    s, c = torch.sin(w * rcl), torch.cos(w * rcl)
    b = norm * s / rcl
    db = norm * (w * c / rcl - s / (rcl * rcl))
    x = (r / rc)[:, None]
    a0, a1, a2 = -(p + 1) * (p + 2) / 2.0, p * (p + 2.0), -p * (p + 1) / 2.0
    xp = x ** p
    env = 1.0 + xp * (a0 + x * (a1 + a2 * x))
    denv = (xp / x.clamp(min=1e-30)) * (p * a0 + x * ((p + 1) * a1 + (p + 2) * a2 * x)) / rc
    inside = (r < rc)[:, None].to(r.dtype)
    return b * env * inside, (db * env + b * denv) * inside


def _kernels(t: Tensor) -> bool:
    return t.is_cuda and _ext.cuda_available()


def _basis(r: Tensor, spec) -> Tensor:
    if _kernels(r):
        return _ext.ops().radial_basis(r.contiguous(), spec.freqs.to(r.device), spec.norm, spec.rc, spec.p)
    rad, drad = bessel_envelope(r, spec.freqs.to(r), spec.norm, spec.rc, spec.p)
    return torch.cat([rad, drad], 0)


def _act(A: Tensor, c: float) -> Tensor:
    if _kernels(A):
        return _ext.ops().radial_act(A, c)
    E = A.shape[0] // 2
    a, ad = A[:E], A[E:]
    f, f1, _ = _silu_d(a)
    return torch.cat([c * f, c * f1 * ad], 0)


def _dact(A: Tensor, dH: Tensor, c: float, primal_only: bool, want_H: bool):
    """Reverse of :func:`_act`: ``DA`` and optionally the forward activations ``H``."""
    if _kernels(A):
        DA, H = _ext.ops().radial_dact(A, dH.contiguous(), c, primal_only, want_H)
        return DA, (H if want_H else None)
    E = A.shape[0] // 2
    a, ad = A[:E], A[E:]
    f, f1, f2 = _silu_d(a)
    if primal_only:
        return c * dH * f1, (c * f if want_H else None)
    dh, dhd = dH[:E], dH[E:]
    DA = torch.cat([c * (dh * f1 + dhd * f2 * ad), c * dhd * f1], 0)
    H = torch.cat([c * f, c * f1 * ad], 0) if want_H else None
    return DA, H


def _mm(X: Tensor, W: Tensor) -> Tensor:
    return gemm.mm_raw(X.contiguous(), W)


def _mmT(X: Tensor, D: Tensor) -> Tensor:
    """``X^T @ D`` (a reduction over the rows)."""
    return gemm.mm_t_raw(X.contiguous(), D.contiguous())


# ------------------------------------------------------------------------------- network
class RadialSpec:
    """Constants of one folded e3nn MLP: factor and activation constant per layer, column scale."""

    def __init__(self, net, col_scale: Optional[Tensor], freqs: Tensor, norm: float, rc: float, p: int):
        layers = net.folded()
        for _, _, act, _ in layers[:-1]:
            if act is not torch.nn.functional.silu:
                raise NotImplementedError("the fused radial network supports SiLU hidden layers")
        if layers[-1][2] is not None:
            raise NotImplementedError("the fused radial network has a linear output layer")
        self.factors = [float(f) for _, f, _, _ in layers]
        self.consts = [float(c) for _, _, _, c in layers[:-1]]
        self.col_scale = col_scale
        self.freqs, self.norm, self.rc, self.p = freqs, float(norm), float(rc), int(p)


def _eff(Ws: Sequence[Tensor], spec: RadialSpec) -> List[Tensor]:
    out = [W * f for W, f in zip(Ws, spec.factors)]
    if spec.col_scale is not None:
        out[-1] = out[-1] * spec.col_scale
    return out


def _forward(r: Tensor, We: List[Tensor], spec: RadialSpec):
    E = r.shape[0]
    H0 = _basis(r, spec)                          # (2E, n) stacked basis and its derivative
    H = H0
    acts = []
    for k in range(len(We) - 1):
        A = _mm(H, We[k])
        H = _act(A, spec.consts[k])
        acts.append(A)
    out = _mm(H, We[-1])
    return out[:E], out[E:], acts, H0


def _reverse(E: int, We: List[Tensor], spec: RadialSpec, acts: List[Tensor], H0: Tensor,
             dR: Optional[Tensor], dRd: Optional[Tensor]) -> List[Tensor]:
    """Effective-weight gradients for cotangents ``dR`` (primal rows) and ``dRd`` (tangent rows)."""
    primal = dRd is None
    if primal:
        D = dR
    elif (dR is not None and dR.is_contiguous() and dRd.is_contiguous() and dR.shape == dRd.shape
          and dRd.data_ptr() == dR.data_ptr() + dR.numel() * dR.element_size()):
        D = dR.as_strided((2 * dR.shape[0],) + tuple(dR.shape[1:]), dR.stride())   # adjacent: no copy
    else:
        D = torch.cat([dR if dR is not None else torch.zeros_like(dRd), dRd], 0)
    grads: List[Optional[Tensor]] = [None] * len(We)
    dH = _mm(D, We[-1].t())
    # activations of the last hidden layer (input of the output layer)
    k = len(acts) - 1
    DA, Hk = _dact(acts[k], dH, spec.consts[k], primal, True)
    grads[-1] = _mmT(Hk, D)
    for k in range(len(acts) - 1, -1, -1):
        if k > 0:
            DA_prev_in = _mm(DA, We[k].t())
            DAn, Hp = _dact(acts[k - 1], DA_prev_in, spec.consts[k - 1], primal, True)
            grads[k] = _mmT(Hp, DA)
            DA = DAn
        else:
            Hin = H0[:E] if primal else H0
            grads[0] = _mmT(Hin, DA)
    return grads


def _raw_grads(gE: List[Tensor], spec: RadialSpec) -> List[Tensor]:
    out = [g * f for g, f in zip(gE, spec.factors)]
    if spec.col_scale is not None:
        out[-1] = out[-1] * spec.col_scale
    return out


class _Radial(Function):
    @staticmethod
    def forward(ctx, r, spec, *Ws):
        We = _eff(Ws, spec)
        R, Rd, acts, H0 = _forward(r, We, spec)
        ctx.spec = spec
        ctx.save_for_backward(r, Rd, H0, *acts, *Ws)
        ctx.n_acts = len(acts)
        return R

    @staticmethod
    def backward(ctx, gR):
        saved = ctx.saved_tensors
        r, Rd, H0 = saved[:3]
        acts = list(saved[3:3 + ctx.n_acts])
        Ws = list(saved[3 + ctx.n_acts:])
        spec = ctx.spec
        g_r = None
        if ctx.needs_input_grad[0] and not MODES.params_only:
            g_r = _RadialVJP.apply(gR, r, Rd, H0, spec, len(acts), *acts, *Ws)
        gW = [None] * len(Ws)
        if any(ctx.needs_input_grad[2:]) and not MODES.force_pass:
            with torch.no_grad():
                We = _eff(Ws, spec)
                gE = _reverse(r.shape[0], We, spec, acts, H0, gR.contiguous(), None)
                gW = _raw_grads(gE, spec)
        return (g_r, None, *gW)


class _RadialVJP(Function):
    """``g_r[e] = sum_j gR[e, j] dR/dr[e, j]`` and its derivatives."""

    @staticmethod
    def forward(ctx, gR, r, Rd, H0, spec, n_acts, *rest):
        acts = rest[:n_acts]
        Ws = rest[n_acts:]
        ctx.spec, ctx.n_acts = spec, n_acts
        ctx.save_for_backward(gR, r, Rd, H0, *acts, *Ws)
        return (gR * Rd).sum(-1)

    @staticmethod
    @once_differentiable
    def backward(ctx, u):
        saved = ctx.saved_tensors
        gR, r, Rd, H0 = saved[:4]
        acts = list(saved[4:4 + ctx.n_acts])
        Ws = list(saved[4 + ctx.n_acts:])
        spec = ctx.spec
        n_in = 6 + len(acts)
        cot_gR = u[:, None] * Rd if ctx.needs_input_grad[0] else None
        gW = [None] * len(Ws)
        if any(ctx.needs_input_grad[n_in:]):
            We = _eff(Ws, spec)
            gE = _reverse(r.shape[0], We, spec, acts, H0, None, (u[:, None] * gR).contiguous())
            gW = _raw_grads(gE, spec)
        cot_r = None
        if ctx.needs_input_grad[1] and not MODES.params_only:
            # d/dr of sum gR dR/dr: second derivative along r, by autograd on the PyTorch formulas
            with torch.enable_grad():
                rr = r.detach().requires_grad_(True)
                We = _eff([w.detach() for w in Ws], spec)
                rad, drad = bessel_envelope(rr, spec.freqs.to(rr), spec.norm, spec.rc, spec.p)
                H = torch.cat([rad, drad], 0)
                E = rr.shape[0]
                for k in range(len(We) - 1):
                    A = H @ We[k]
                    f, f1, _ = _silu_d(A[:E])
                    H = torch.cat([spec.consts[k] * f, spec.consts[k] * f1 * A[E:]], 0)
                Rd2 = (H @ We[-1])[E:]
                (cot_r,) = torch.autograd.grad((gR * Rd2).sum(-1), rr, u)
        return (cot_gR, cot_r, None, None, None, None) + (None,) * len(acts) + tuple(gW)


def radial_network(r: Tensor, net, col_scale: Optional[Tensor], freqs: Tensor, norm: float, rc: float,
                   p: int) -> Tensor:
    """``R (E, n_out)`` of the enveloped-Bessel MLP at edge lengths ``r (E,)`` (see module notes)."""
    spec = RadialSpec(net, col_scale, freqs, norm, rc, p)
    Ws = [layer.weight for layer in net]
    return _Radial.apply(r, spec, *Ws)
