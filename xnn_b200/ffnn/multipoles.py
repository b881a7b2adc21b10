"""Polarizable multipole electrostatics with smooth particle-mesh Ewald (AMOEBA-style).

Sites carry charges ``q``, dipoles ``d`` (e A) and traceless quadrupoles ``Q`` (e A^2) in the
global frame, and isotropic polarizabilities ``alpha_pol`` (A^3). The electrostatic energy of a
periodic set of multipoles (eV) is the Ewald sum

    E = E_real + E_recip + E_self (+ the neutralising-background term of a net charge),

where the interaction of two sites is the operator ``L_i L_j g(|r_j - r_i|)`` with
``L = q + d . grad + (1/3) Q : grad grad`` acting on each site's own position, ``g`` the
erfc-screened Coulomb kernel in real space (cutoff ``rc``) and the Gaussian-smoothed rest in
reciprocal space. Pairs of one molecule (``molecule`` ids) are excluded from every interaction;
their reciprocal-space share is removed with the ``erf`` kernel.

Reciprocal space is smooth PME (Essmann et al., J. Chem. Phys. 103, 8577 (1995)): the operator
``L`` is applied to the order-``p`` cardinal B-spline weights of each site (first and second
spline derivatives, mapped to Cartesian axes by the reciprocal cell), spread on a ``K1 x K2 x
K3`` mesh, transformed by a real FFT and weighted by ``exp(-pi^2 m^2 / a^2) / (pi V m^2) B(m)``
with the Euler exponential-spline moduli ``B``. Forces and fields follow by differentiation.

Induced dipoles minimise ``U(mu) = E(q, d + mu, Q) + sum |mu_i|^2 / (2 alpha_i)``, where every
interaction involving ``mu`` uses Thole-damped real-space kernels (``a = 0.39``, ``u = r /
(alpha_i alpha_j)^(1/6)``, as AMOEBA damps induction) and the permanent multipoles interact
undamped; the stationary point solves ``(alpha^-1 - T) mu = F_perm`` by preconditioned
conjugate gradients (Jacobi),
``T mu`` being the field of the dipoles ``mu`` (one spread, FFT and back-interpolation per
iteration). At convergence the forces are ``-dU/dr`` at fixed ``mu`` (stationarity).

Real-space pair terms follow the B_n formalism (B_0 = g, B_n = -(1/r) dB_{n-1}/dr) with the
five contraction terms of the Tinker multipole code family; the Ewald self terms of charges,
dipoles and quadrupoles are included. Everything is differentiable tensor code (CUDA or CPU);
the mesh can be split over processes as z-slabs (:mod:`xnn_b200.ffnn.slab_fft`).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
from torch import Tensor, nn

#: Coulomb constant (eV A / e^2) and one Debye in e A
KE = 14.399645478425668
DEBYE = 0.20819433622621843
#: two sites of one molecule closer than this (A) interact only through the molecule's exclusion
MOLECULE_REACH = 3.0


# ----------------------------------------------------------------------------- B-splines
def _spline_padded(t: Tensor, n: int, p: int) -> Tensor:
    """``M_n(t + j)`` for ``j = 0..p-1`` (zero for ``j >= n``), ``(..., p)``."""
    w = [t, 1.0 - t]
    for m in range(3, n + 1):
        new = []
        for j in range(m):
            v = torch.zeros_like(t)
            if j < m - 1:
                v = v + (t + j) / (m - 1) * w[j]
            if j >= 1:
                v = v + (m - t - j) / (m - 1) * w[j - 1]
            new.append(v)
        w = new
    w = w + [torch.zeros_like(t)] * (p - len(w))
    return torch.stack(w[:p], -1)


def bspline_derivs(t: Tensor, p: int) -> Tuple[Tensor, Tensor, Tensor]:
    """``M_p``, ``M_p'`` and ``M_p''`` at ``t + j`` (``j = 0..p-1``), each ``(..., p)``; the site
    spreads onto grid points ``floor(u) - j``."""
    m0 = _spline_padded(t, p, p)
    a1 = _spline_padded(t, p - 1, p)
    a2 = _spline_padded(t, p - 2, p)
    sh = lambda a, k: torch.cat([torch.zeros_like(a[..., :k]), a[..., :p - k]], -1)  # noqa: E731
    m1 = a1 - sh(a1, 1)
    m2 = a2 - 2.0 * sh(a2, 1) + sh(a2, 2)
    return m0, m1, m2


def bspline_moduli(K: int, p: int, dtype, device) -> Tensor:
    """``|b(m)|^2`` of the Euler exponential spline for the ``K`` FFT frequencies."""
    mk = _spline_padded(torch.zeros((), dtype=torch.float64), p, p)        # M_p(j), j = 0..p-1
    coef = mk[1:p]                                                          # M_p(1..p-1)
    m = torch.arange(K, dtype=torch.float64)
    k = torch.arange(0, p - 1, dtype=torch.float64)
    ang = 2.0 * math.pi * m[:, None] * k[None, :] / K
    re = (coef[None, :] * torch.cos(ang)).sum(1)
    im = (coef[None, :] * torch.sin(ang)).sum(1)
    den = re * re + im * im
    bad = den < 1e-10
    if bool(bad.any()):
        idx = torch.nonzero(bad).flatten()
        for i in idx.tolist():
            den[i] = 0.5 * (den[(i - 1) % K] + den[(i + 1) % K])
    return (1.0 / den).to(dtype=dtype, device=device)


def _freq(K: int, device) -> Tensor:
    return torch.fft.fftfreq(K, d=1.0 / K, device=device)


# ----------------------------------------------------------------------------- reciprocal
def spline_stencil(pos: Tensor, cell: Tensor, mesh: List[int], p: int):
    """Per site: base grid index ``floor(u)`` ``(n, 3)`` and per-axis spline values / first /
    second derivatives ``(n, 3, p)``, plus ``G (3, 3)`` with ``du_a / dr_b = G[b, a]``."""
    inv = torch.linalg.inv(cell)
    K = torch.tensor(mesh, dtype=pos.dtype, device=pos.device)
    u = (pos @ inv) * K
    base = torch.floor(u.detach())
    t = u - base
    m0, m1, m2 = bspline_derivs(t, p)
    G = inv * K[None, :]
    return base.long(), m0, m1, m2, G


class _SpreadKernel(torch.autograd.Function):
    """Spreading on the CUDA kernel (``csrc/pme_spread.cu``) into a float32 mesh; the backward
    is the gather kernel (fields and forces). Differentiable in positions and dipoles."""

    @staticmethod
    def forward(ctx, pos, d, cell, q, Q, mesh, p, z0, nz):
        from .. import _ext
        K = torch.tensor(mesh, dtype=torch.float64, device=pos.device)
        G = (torch.linalg.inv(cell.detach().double()) * K[None, :]).contiguous()
        args = (pos.detach().contiguous(), G, list(mesh), int(p), int(z0), int(nz),
                None if q is None else q.detach().contiguous(), None if d is None else d.detach().contiguous(),
                None if Q is None else Q.detach().reshape(-1, 9).contiguous())
        ctx.args = args
        return _ext.ops().pme_spread(*args)

    @staticmethod
    def backward(ctx, phi):
        from .. import _ext
        want_p, want_d = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        gd, gp = _ext.ops().pme_gather(*ctx.args, phi.float().contiguous(), bool(want_d), bool(want_p))
        return (gp if want_p else None, gd if want_d else None) + (None,) * 7


def spread(pos: Tensor, cell: Tensor, q: Optional[Tensor], d: Optional[Tensor], Q: Optional[Tensor],
           mesh: List[int], p: int, z_range: Optional[Tuple[int, int]] = None,
           out_dtype: Optional[torch.dtype] = None) -> Tensor:
    """Mesh of ``sum_i L_i W_i`` (``(K1, K2, K3)``; with ``z_range`` only planes ``[z0, z1)``
    of the third axis, ``(K1, K2, z1 - z0)``). For a float32 mesh of float64 CUDA sites the
    spreading kernel runs (its adjoint differentiates positions and dipoles; derivatives in the
    charges, quadrupoles or cell take the tensor formulas)."""
    n = pos.shape[0]
    others = torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (q, Q, cell))
    if (out_dtype == torch.float32 and pos.is_cuda and pos.dtype == torch.float64 and 4 <= p <= 6 and _kernel_ok()
            and not others and hasattr(__import__("xnn_b200._ext", fromlist=["ops"]).ops(), "pme_spread")):
        z0, z1 = z_range if z_range is not None else (0, mesh[2])
        return _SpreadKernel.apply(pos, d, cell, q, Q, list(mesh), p, z0, z1 - z0)
    K1, K2, K3 = mesh
    base, m0, m1, m2, G = spline_stencil(pos, cell, mesh, p)
    # multipoles in scaled-fractional coordinates: d_u = G^T d, Q_u = G^T Q G
    coef0 = q if q is not None else pos.new_zeros(n)
    du = (d[:, :, None] * G[None]).sum(1) if d is not None else None
    Qu = ((G[None, :, :, None, None] * Q[:, :, None, :, None] * G[None, None, None, :, :]).sum((1, 3))
          if Q is not None else None)                                       # G^T Q G per site
    j = torch.arange(p, device=pos.device)
    ix = (base[:, 0, None] - j[None, :]) % K1
    iy = (base[:, 1, None] - j[None, :]) % K2
    iz = (base[:, 2, None] - j[None, :]) % K3
    a0, b0, c0 = m0[:, 0], m0[:, 1], m0[:, 2]
    a1, b1, c1 = m1[:, 0], m1[:, 1], m1[:, 2]
    val = coef0[:, None, None, None] * a0[:, :, None, None] * b0[:, None, :, None] * c0[:, None, None, :]
    if du is not None:
        val = val + du[:, 0, None, None, None] * a1[:, :, None, None] * b0[:, None, :, None] * c0[:, None, None, :]
        val = val + du[:, 1, None, None, None] * a0[:, :, None, None] * b1[:, None, :, None] * c0[:, None, None, :]
        val = val + du[:, 2, None, None, None] * a0[:, :, None, None] * b0[:, None, :, None] * c1[:, None, None, :]
    if Qu is not None:
        a2, b2, c2 = m2[:, 0], m2[:, 1], m2[:, 2]
        fa = [a0, a1, a2]
        fb = [b0, b1, b2]
        fc = [c0, c1, c2]
        for x in range(3):
            for y in range(3):
                order = [0, 0, 0]
                order[x] += 1
                order[y] += 1
                w = Qu[:, x, y] / 3.0
                val = val + w[:, None, None, None] * fa[order[0]][:, :, None, None] * \
                    fb[order[1]][:, None, :, None] * fc[order[2]][:, None, None, :]
    flat_xy = (ix[:, :, None] * K2 + iy[:, None, :])                       # (n, p, p)
    if z_range is None:
        idx = flat_xy[:, :, :, None] * K3 + iz[:, None, None, :]
        grid = pos.new_zeros(K1 * K2 * K3).index_add_(0, idx.reshape(-1), val.reshape(-1))
        return grid.view(K1, K2, K3)
    z0, z1 = z_range
    nz = z1 - z0
    keep = (iz >= z0) & (iz < z1)
    idx = flat_xy[:, :, :, None] * nz + (iz - z0).clamp(0, max(nz - 1, 0))[:, None, None, :]
    val = val * keep[:, None, None, :].to(val.dtype)
    grid = pos.new_zeros(K1 * K2 * nz).index_add_(0, idx.reshape(-1), val.reshape(-1))
    return grid.view(K1, K2, nz)


def gather_dipole_gradient(pos: Tensor, cell: Tensor, d: Tensor, mesh: List[int], p: int,
                           z_range: Tuple[int, int], phi: Tensor) -> Tensor:
    """``dE/dd`` of the spread dipoles for a mesh potential ``phi = dE/dgrid`` on the planes
    ``z_range`` (the spreading's adjoint): the gather kernel on CUDA (float64 sites, float32 mesh),
    autograd through the spreading formulas otherwise."""
    z0, z1 = z_range
    if (pos.is_cuda and pos.dtype == torch.float64 and phi.dtype == torch.float32 and 4 <= p <= 6
            and _kernel_ok()):
        from .. import _ext
        K = torch.tensor(mesh, dtype=torch.float64, device=pos.device)
        G = (torch.linalg.inv(cell.detach().double()) * K[None, :]).contiguous()
        gd, _ = _ext.ops().pme_gather(pos.detach().contiguous(), G, list(mesh), int(p), int(z0), int(z1 - z0),
                                      None, d.detach().contiguous(), None, phi.contiguous(), True, False)
        return gd
    dd = d.detach().clone().requires_grad_(True)
    with torch.enable_grad():
        grid = spread(pos.detach(), cell.detach(), None, dd, None, list(mesh), p, z_range=z_range)
        (g,) = torch.autograd.grad((grid * phi.to(grid.dtype)).sum(), dd)
    return g


def influence(cell: Tensor, mesh: List[int], alpha: float, p: int, dtype, device) -> Tensor:
    """``exp(-pi^2 m^2 / alpha^2) / (pi V m^2) B(m)`` on the rfft half-spectrum ``(K1, K2, K3//2+1)``,
    zero at ``m = 0`` and doubled where the half spectrum stands for two conjugate terms."""
    K1, K2, K3 = mesh
    rec = torch.linalg.inv(cell).t().to(torch.float64)                      # rows: reciprocal vectors
    f1, f2 = _freq(K1, device).double(), _freq(K2, device).double()
    f3 = torch.arange(K3 // 2 + 1, device=device, dtype=torch.float64)
    m = (f1[:, None, None, None] * rec[0] + f2[None, :, None, None] * rec[1] + f3[None, None, :, None] * rec[2])
    m2 = (m * m).sum(-1)
    vol = torch.det(cell.to(torch.float64)).abs()
    B = (bspline_moduli(K1, p, torch.float64, device)[:, None, None] * bspline_moduli(K2, p, torch.float64, device)[
        None, :, None] * bspline_moduli(K3, p, torch.float64, device)[None, None, :K3 // 2 + 1])
    with torch.no_grad():
        safe = torch.where(m2 > 0, m2, torch.ones_like(m2))
    val = torch.exp(-math.pi ** 2 * m2 / alpha ** 2) / (math.pi * vol * safe) * B
    val = torch.where(m2 > 0, val, torch.zeros_like(val))
    w = torch.full((K3 // 2 + 1,), 2.0, dtype=torch.float64, device=device)
    w[0] = 1.0
    if K3 % 2 == 0:
        w[-1] = 1.0
    return (val * w[None, None, :]).to(dtype)


def recip_energy(grid: Tensor, infl: Tensor) -> Tensor:
    """``(1/2) sum_m infl(m) |F(Q)(m)|^2`` (Coulomb units) of a full mesh."""
    F = torch.fft.rfftn(grid)
    return 0.5 * (infl * (F.real * F.real + F.imag * F.imag)).sum()


# ----------------------------------------------------------------------------- real space
def _bn(r: Tensor, alpha: float, kind: str, nmax: int = 4) -> List[Tensor]:
    """``B_0..B_nmax`` of ``erfc(a r)/r`` (``kind="erfc"``) or ``-erf(a r)/r`` (``"neg_erf"``)."""
    r2 = r * r
    if kind == "erfc":
        b = [torch.erfc(alpha * r) / r]
        ex = torch.exp(-alpha * alpha * r2)
        f = 1.0 / (alpha * math.sqrt(math.pi))
        for n in range(1, nmax + 1):
            f = f * 2.0 * alpha * alpha
            b.append(((2 * n - 1) * b[-1] + f * ex) / r2)
        return b
    c = _bn(r, alpha, "erfc", nmax)
    inv = [1.0 / r]
    for n in range(1, nmax + 1):
        inv.append((2 * n - 1) * inv[-1] / r2)
    return [ci - vi for ci, vi in zip(c, inv)]          # erfc/r - 1/r = -erf/r


def pair_energy(v: Tensor, qi, di, Qi, qj, dj, Qj, B: List[Tensor]) -> Tensor:
    """``L_i L_j g`` per pair with ``v = r_j - r_i`` and ``B_n`` of ``g`` (Tinker-scaled Q' = Q/3)."""
    Qi3, Qj3 = Qi / 3.0, Qj / 3.0
    dri, drk = (di * v).sum(-1), (dj * v).sum(-1)
    # 3x3 products written out elementwise (batched tiny matmuls are slow library calls)
    qir = (Qi3 * v[..., None, :]).sum(-1)
    qkr = (Qj3 * v[..., None, :]).sum(-1)
    qrri, qrrk = (qir * v).sum(-1), (qkr * v).sum(-1)
    qrrik = (qir * qkr).sum(-1)
    qik = (Qi3 * Qj3).sum((-1, -2))
    dik = (di * dj).sum(-1)
    diqkr = (di * qkr).sum(-1)
    dkqir = (dj * qir).sum(-1)
    t1 = qi * qj
    t2 = qj * dri - qi * drk + dik
    t3 = qi * qrrk + qj * qrri - dri * drk + 2.0 * (dkqir - diqkr + qik)
    t4 = dri * qrrk - drk * qrri - 4.0 * qrrik
    t5 = qrri * qrrk
    return t1 * B[0] + t2 * B[1] + t3 * B[2] + t4 * B[3] + t5 * B[4]


def _kernel_ok() -> bool:
    from .. import _ext
    return _ext.cuda_available() and hasattr(_ext.ops(), "mp_real")


def _shift_vec(shift: Tensor, cell: Tensor) -> Tensor:
    """``shift @ cell`` for integer shifts (three scaled rows, no library matmul)."""
    sf = shift.to(cell.dtype)
    return sf[:, 0:1] * cell[0] + sf[:, 1:2] * cell[1] + sf[:, 2:3] * cell[2]


def thole_damp(B: List[Tensor], r: Tensor, au3: Tensor) -> List[Tensor]:
    """Thole-damped ``B_1..B_3`` (``au3 = a (r / (alpha_i alpha_j)^(1/6))^3``): the bare ``1/r^n``
    parts scaled by ``lambda_3, lambda_5, lambda_7`` (AMOEBA's damping of induction)."""
    ex = torch.exp(-au3)
    l3 = 1.0 - ex
    l5 = 1.0 - (1.0 + au3) * ex
    l7 = 1.0 - (1.0 + au3 + 0.6 * au3 * au3) * ex
    r2 = r * r
    r3 = r2 * r
    return [B[0], B[1] - (1.0 - l3) / r3, B[2] - 3.0 * (1.0 - l5) / (r3 * r2),
            B[3] - 15.0 * (1.0 - l7) / (r3 * r2 * r2), B[4]]


class _RealKernel(torch.autograd.Function):
    """Real-space pair sum on the CUDA kernel (``csrc/multipole_real.cu``); first derivatives
    with respect to positions and dipoles (forces and fields)."""

    @staticmethod
    def forward(ctx, pos, d, cell, q, Q, pol, i, j, shift, excluded, alpha, thole):
        from .. import _ext
        e, gp, gd = _ext.ops().mp_real(pos.contiguous(), cell.contiguous(), q.contiguous(), d.contiguous(),
                                       Q.contiguous(), pol.contiguous(), i.contiguous(), j.contiguous(),
                                       shift.contiguous(), excluded.contiguous(), float(alpha),
                                       float(thole) if thole is not None else -1.0,
                                       ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        ctx.save_for_backward(gp if ctx.needs_input_grad[0] else None, gd if ctx.needs_input_grad[1] else None)
        return e[0]

    @staticmethod
    def backward(ctx, g):
        gp, gd = ctx.saved_tensors
        return (None if gp is None else g * gp, None if gd is None else g * gd) + (None,) * 10


def real_energy(pos: Tensor, cell: Tensor, i: Tensor, j: Tensor, shift: Tensor, excluded: Tensor,
                q: Tensor, d: Tensor, Q: Tensor, alpha: float, chunk: int = 1 << 21,
                pol: Optional[Tensor] = None, thole: Optional[float] = None) -> Tensor:
    """Sum over unique pairs ``(i, j, shift)`` (``v = pos[j] - pos[i] + shift @ cell``); excluded
    pairs contribute ``-erf`` (their reciprocal share removed); with ``thole`` the dipole,
    dipole-dipole and dipole-quadrupole kernels are Thole-damped. On CUDA (float64) the pair
    kernel evaluates it (differentiable in positions and dipoles)."""
    # the pair kernel differentiates positions and dipoles; derivatives in the charges, the
    # quadrupoles (frame torques) or the cell (stress) take the tensor formulas below
    others = torch.is_grad_enabled() and (q.requires_grad or Q.requires_grad or cell.requires_grad)
    if pos.is_cuda and pos.dtype == torch.float64 and _kernel_ok() and not others:
        pw = pol if pol is not None else torch.ones_like(q)
        return _RealKernel.apply(pos, d, cell, q, Q.reshape(-1, 9), pw, i, j, shift, excluded, alpha, thole)
    e = pos.new_zeros(())
    for s in range(0, i.shape[0], chunk):
        a, b = i[s:s + chunk], j[s:s + chunk]
        v = pos[b] - pos[a] + _shift_vec(shift[s:s + chunk], cell)
        r = torch.linalg.norm(v, dim=-1)
        ex = excluded[s:s + chunk]
        Bc = _bn(r, alpha, "erfc")
        if thole is not None:
            u = r / (pol[a] * pol[b]) ** (1.0 / 6.0)
            Bc = thole_damp(Bc, r, thole * u * u * u)
        Be = _bn(r, alpha, "neg_erf")
        B = [torch.where(ex, y, x) for x, y in zip(Bc, Be)]
        e = e + pair_energy(v, q[a], d[a], Q[a], q[b], d[b], Q[b], B).sum()
    return e


def intra_dipole_energy(pos: Tensor, cell: Tensor, pairs, mu: Tensor, pol: Tensor, thole: Optional[float]) -> Tensor:
    """Dipole-dipole energy (Coulomb units) of the excluded (intramolecular) pairs with the bare,
    Thole-damped kernel: added to a sum in which those pairs contribute nothing, it makes the
    induced dipoles of a molecule interact in full."""
    i, j, sh, ex = pairs
    if not bool(ex.any()):
        return pos.new_zeros(())
    a, b, s_ = i[ex], j[ex], sh[ex]
    v = pos[b] - pos[a] + _shift_vec(s_, cell)
    r = torch.linalg.norm(v, dim=-1)
    r2 = r * r
    B = [1.0 / r, 1.0 / (r2 * r), 3.0 / (r2 * r2 * r), 15.0 / (r2 * r2 * r2 * r), 105.0 / (r2 * r2 * r2 * r2 * r)]
    if thole is not None:
        u = r / (pol[a] * pol[b]) ** (1.0 / 6.0)
        B = thole_damp(B, r, thole * u * u * u)
    z = mu.new_zeros(a.shape[0])
    z3 = mu.new_zeros(a.shape[0], 3, 3)
    return pair_energy(v, z, mu[a], z3, z, mu[b], z3, B).sum()


def self_energy(q: Tensor, d: Tensor, Q: Tensor, alpha: float) -> Tensor:
    a2 = 2.0 * alpha * alpha
    Q3 = Q / 3.0
    return -(alpha / math.sqrt(math.pi)) * ((q * q).sum() + a2 * ((d * d).sum() / 3.0 + 2.0 * a2 * (Q3 * Q3).sum() / 5.0))


def background_energy(q: Tensor, cell: Tensor, alpha: float) -> Tensor:
    vol = torch.det(cell).abs()
    return -math.pi * q.sum() ** 2 / (2.0 * vol * alpha * alpha)


# ----------------------------------------------------------------------------- pair list
def multipole_pairs(pos: Tensor, cell: Tensor, cutoff: float, molecule: Optional[Tensor],
                    receivers: Optional[Tuple[int, int]] = None):
    """Unique pairs within ``cutoff`` (every unordered pair, and an atom with a nonzero image of
    itself, once), their shifts, and which pairs belong to one molecule (excluded).

    Of the two directed edges of a pair the one kept is ``src < dst`` when ``src + dst`` is odd
    and ``src > dst`` when it is even (an image of itself: the positive shift), so the pairs kept
    by a receiving atom are about half of its neighbours whatever its index. With ``receivers``
    only edges into those atoms are searched: processes that split the atoms into ranges get
    disjoint, balanced shares of the pairs from their own searches."""
    from ..data.neighborlist import build_neighbor_list
    ei, sh = build_neighbor_list(pos.detach().double(), cutoff, cell.detach().double(),
                                 torch.ones(3, dtype=torch.bool), receivers=receivers)
    src, dst = ei[0], ei[1]
    # edge vector pos[dst] - pos[src] + sh @ cell; keep each unordered pair once
    odd = ((src + dst) % 2) == 1
    positive = (sh[:, 0] > 0) | ((sh[:, 0] == 0) & ((sh[:, 1] > 0) | ((sh[:, 1] == 0) & (sh[:, 2] > 0))))
    key = torch.where(src == dst, positive, torch.where(odd, src < dst, src > dst))
    i, j, s = src[key], dst[key], sh[key]
    if molecule is None:
        excluded = torch.zeros_like(i, dtype=torch.bool)
    else:
        # the pairs of one molecule (its minimal image: molecules are far smaller than the box)
        p64, c64 = pos.detach().double(), cell.detach().double()
        r = torch.linalg.norm(p64[j.to(pos.device)] - p64[i.to(pos.device)] + s.to(pos.device).double() @ c64, dim=-1)
        m = molecule.to(pos.device)
        excluded = (m[i.to(pos.device)] == m[j.to(pos.device)]) & (r < MOLECULE_REACH)
    return i.to(pos.device), j.to(pos.device), s.to(pos.device), excluded.to(pos.device)


# ----------------------------------------------------------------------------- dipole operator
class DipoleOperator:
    """``T v``: the field (Coulomb units) that a set of dipoles ``v`` produces at every site, with
    the induction's Thole damping (``pol`` given) -- the matrix of the induced-dipole solve,
    applied without an energy graph.

    * real space: per pair ``-[B_1 v_j - B_2 (v_j . r) r]`` (and symmetrically), ``B_1, B_2`` of the
      screened (or, within a molecule, ``-erf``) kernel formed once (``csrc/pme_induce.cu``);
    * reciprocal space: the dipoles spread on the mesh, the FFT convolution, and the gather of
      ``-dE/dv`` (the spreading kernel's adjoint);
    * self term: ``4 a^3 / (3 sqrt(pi)) v``.

    With the work split over processes each returns its share, summed over the group."""

    def __init__(self, mod: "PolarizableMultipoles", pos: Tensor, cell: Tensor, pairs, pol: Optional[Tensor]):
        self.mod = mod
        self.pos, self.cell = pos.detach(), cell.detach()
        i, j, sh, ex = pairs
        self.i, self.j = i, j
        s = mod.setup
        a = s.alpha
        self.self_coef = 4.0 * a ** 3 / (3.0 * math.sqrt(math.pi)) if mod.rank == 0 else 0.0
        self.kernel = pos.is_cuda and pos.dtype == torch.float64 and _kernel_ok()
        th = mod.thole if pol is not None else None
        pw = (pol if pol is not None else torch.ones(pos.shape[0], dtype=pos.dtype, device=pos.device)).detach()
        if self.kernel:
            from .. import _ext
            self.v, self.b1, self.b2 = _ext.ops().dipole_pairs(
                self.pos.contiguous(), self.cell.contiguous(), i.contiguous(), j.contiguous(), sh.contiguous(),
                ex.contiguous(), pw.contiguous(), float(a), float(th) if th is not None else -1.0)
        else:
            v = self.pos[j] - self.pos[i] + _shift_vec(sh, self.cell)
            r = torch.linalg.norm(v, dim=-1)
            Bc = _bn(r, a, "erfc", 2)
            b1, b2 = Bc[1], Bc[2]
            if th is not None:
                u = r / (pw[i] * pw[j]) ** (1.0 / 6.0)
                au3 = th * u * u * u
                e = torch.exp(-au3)
                r3 = r * r * r
                b1 = b1 - e / r3                               # (1 - lambda_3) / r^3
                b2 = b2 - 3.0 * (1.0 + au3) * e / (r3 * r * r)  # 3 (1 - lambda_5) / r^5
            Be = _bn(r, a, "neg_erf", 2)
            self.v = v
            self.b1 = torch.where(ex, Be[1], b1)
            self.b2 = torch.where(ex, Be[2], b2)

    def _csr(self):
        """The pairs twice, ordered by receiving site (built once per solve): the warp-per-site
        product needs no atomics."""
        if not hasattr(self, "_rows"):
            n = self.pos.shape[0]
            recv = torch.cat([self.i, self.j])
            order = torch.sort(recv, stable=True)[1]
            pair = order % self.i.shape[0]
            ptr = torch.zeros(n + 1, dtype=torch.long, device=recv.device)
            ptr[1:] = torch.cumsum(torch.bincount(recv, minlength=n), 0)
            partner = torch.cat([self.j, self.i]).index_select(0, order).to(torch.int32)
            self._rows = (ptr, partner, self.v.index_select(0, pair).contiguous(),
                          self.b1.index_select(0, pair).contiguous(), self.b2.index_select(0, pair).contiguous())
        return self._rows

    def real(self, d: Tensor) -> Tensor:
        if self.kernel:
            from .. import _ext
            ptr, partner, v, b1, b2 = self._csr()
            return _ext.ops().dipole_csr_matvec(ptr, partner, v, b1, b2, d.contiguous())
        v, b1, b2 = self.v, self.b1[:, None], self.b2[:, None]
        dj, di = d[self.j], d[self.i]
        fi = -(b1 * dj - b2 * (dj * v).sum(-1, keepdim=True) * v)
        fj = -(b1 * di - b2 * (di * v).sum(-1, keepdim=True) * v)
        return torch.zeros_like(d).index_add_(0, self.i, fi).index_add_(0, self.j, fj)

    def _direct_setup(self) -> bool:
        """The reciprocal field without an energy graph: one process, CUDA float64 sites and a
        float32 mesh (the spreading and gather kernels)."""
        s = self.mod.setup
        ok = (self.kernel and self.mod.mesh_backend is None and s.fft_dtype == torch.float32 and 4 <= s.order <= 6)
        if ok and not hasattr(self, "_G"):
            K = torch.tensor(s.mesh, dtype=torch.float64, device=self.pos.device)
            self._G = (torch.linalg.inv(self.cell.double()) * K[None, :]).contiguous()
            K3 = s.mesh[2]
            w = torch.full((K3 // 2 + 1,), 2.0, dtype=torch.float32, device=self.pos.device)
            w[0] = 1.0
            if K3 % 2 == 0:
                w[-1] = 1.0
            # the influence function without the half-spectrum doubling (irfftn restores the
            # conjugate half), times the mesh size (the unnormalised inverse transform)
            self._infl = self.mod._influence(self.cell) / w * float(math.prod(s.mesh))
        return ok

    def recip(self, d: Tensor) -> Tensor:
        backend = self.mod.mesh_backend
        if backend is not None and hasattr(backend, "dipole_field"):
            return backend.dipole_field(self.pos, self.cell, d, self.mod.setup)
        if self._direct_setup():
            # field = -dE/dd with E = 1/2 sum_m infl(m) |F(m)|^2: spread d, transform, weigh,
            # transform back to the mesh potential dE/dgrid, gather its stencil derivatives
            from .. import _ext
            s = self.mod.setup
            C = _ext.ops()
            pos = self.pos.contiguous()
            dd = d.contiguous()
            K3 = s.mesh[2]
            grid = C.pme_spread(pos, self._G, list(s.mesh), s.order, 0, K3, None, dd, None)
            phi = torch.fft.irfftn(torch.fft.rfftn(grid) * self._infl, s=list(s.mesh))
            gd, _ = C.pme_gather(pos, self._G, list(s.mesh), s.order, 0, K3, None, dd, None, phi.contiguous(),
                                 True, False)
            return -gd
        n = d.shape[0]
        dd = d.detach().clone().requires_grad_(True)
        with torch.enable_grad():
            e = self.mod.recip(self.pos, self.cell, d.new_zeros(n), dd, d.new_zeros(n, 3, 3))
            (g,) = torch.autograd.grad(e, dd)
        return -g

    def __call__(self, d: Tensor) -> Tensor:
        out = self.real(d) + self.recip(d)
        if self.self_coef:
            out = out + self.self_coef * d
        return self.mod._sum(out)


# ----------------------------------------------------------------------------- module
@dataclass
class EwaldSetup:
    alpha: float = 0.4
    cutoff: float = 7.0
    mesh: Tuple[int, int, int] = (128, 128, 128)
    order: int = 5
    fft_dtype: torch.dtype = torch.float32


class PolarizableMultipoles(nn.Module):
    """Energy, forces and induced dipoles of a periodic polarizable multipole system."""

    def __init__(self, setup: EwaldSetup = EwaldSetup(), tol_debye: float = 1e-5, max_iter: int = 100,
                 mesh_backend=None, group=None, thole: Optional[float] = 0.39, mutual_intra: bool = False):
        """``mesh_backend``: a :class:`~xnn_b200.ffnn.slab_fft.SlabFFT` to split the mesh over the
        processes of ``group`` (the real-space pairs are split too, and fields, energies and
        forces summed); ``None`` evaluates everything here. ``mutual_intra``: the induced dipoles
        of one molecule interact with each other (Thole-damped, AMOEBA's mutual scale 1), while
        every interaction of the permanent multipoles within a molecule stays excluded."""
        super().__init__()
        self.mutual_intra = bool(mutual_intra)
        self.setup = setup
        self.tol = float(tol_debye) * DEBYE
        self.max_iter = int(max_iter)
        self.mesh_backend = mesh_backend
        self.group = group
        self.thole = None if thole is None else float(thole)
        dist_on = mesh_backend is not None and torch.distributed.is_available() and torch.distributed.is_initialized()
        self.world = torch.distributed.get_world_size(group) if dist_on else 1
        self.rank = torch.distributed.get_rank(group) if dist_on else 0
        self._infl = None

    def _sum(self, t: Tensor) -> Tensor:
        if self.world > 1:
            t = t.contiguous()
            torch.distributed.all_reduce(t, group=self.group)
        return t

    def pairs(self, pos, cell, molecule):
        """This process's pairs: with the work split, the pairs received by its range of atoms
        (its own neighbour search, no replicated list)."""
        recv = None
        if self.world > 1:
            n = pos.shape[0]
            base, extra = divmod(n, self.world)
            r0 = self.rank * base + min(self.rank, extra)
            recv = (r0, r0 + base + (1 if self.rank < extra else 0))
        return multipole_pairs(pos, cell, self.setup.cutoff, molecule, receivers=recv)

    def _influence(self, cell: Tensor) -> Tensor:
        s = self.setup
        key = (tuple(cell.detach().reshape(-1).tolist()), cell.device)
        if self._infl is None or self._infl[0] != key:
            self._infl = (key, influence(cell.detach(), list(s.mesh), s.alpha, s.order, s.fft_dtype, cell.device))
        return self._infl[1]

    def recip(self, pos, cell, q, d, Q) -> Tensor:
        s = self.setup
        if self.mesh_backend is not None:
            return self.mesh_backend.energy(pos, cell, q, d, Q, s)
        grid = spread(pos, cell, q, d, Q, list(s.mesh), s.order, out_dtype=s.fft_dtype).to(s.fft_dtype)
        return recip_energy(grid, self._influence(cell)).to(pos.dtype)

    def electrostatic(self, pos, cell, pairs, q, d, Q, pol: Optional[Tensor] = None) -> Tensor:
        """Ewald energy in eV (Coulomb constant applied); with ``pol`` the real-space kernels are
        Thole-damped (the induction energy surface)."""
        s = self.setup
        i, j, sh, ex = pairs
        th = self.thole if pol is not None else None
        e = self.recip(pos, cell, q, d, Q) + real_energy(pos, cell, i, j, sh, ex, q, d, Q, s.alpha, pol=pol, thole=th)
        if self.rank == 0:
            e = e + self_energy(q, d, Q, s.alpha) + background_energy(q, cell, s.alpha)
        return KE * e           # this process's share when the work is split

    def polarizable_energy(self, pos, cell, pairs, q, d, Q, pol, mu) -> Tensor:
        """``U(mu)``: permanent multipoles interact undamped, everything involving the induced
        dipoles through the Thole-damped kernels, plus ``sum |mu|^2 / (2 alpha)``."""
        s = self.setup
        i, j, sh, ex = pairs
        u = self.electrostatic(pos, cell, pairs, q, d + mu, Q, pol=pol if self.thole is not None else None)
        if self.thole is not None:
            u = u + KE * (real_energy(pos, cell, i, j, sh, ex, q, d, Q, s.alpha)
                          - real_energy(pos, cell, i, j, sh, ex, q, d, Q, s.alpha, pol=pol, thole=self.thole))
        if self.rank == 0:
            u = u + KE * 0.5 * ((mu * mu).sum(-1) / pol).sum()
        if self.mutual_intra:
            u = u + KE * intra_dipole_energy(pos, cell, pairs, mu, pol, self.thole)
        return u

    def field(self, pos, cell, pairs, q, d, Q, pol: Optional[Tensor] = None) -> Tensor:
        """Electric field ``-dE/d(mu)`` at every site (eV / (e A) units), ``(n, 3)``; Thole-damped
        when ``pol`` is given."""
        mu = torch.zeros_like(d, requires_grad=True)
        with torch.enable_grad():
            e = self.electrostatic(pos.detach(), cell.detach(), pairs, q.detach(), d.detach() + mu, Q.detach(),
                                   pol=pol)
            (g,) = torch.autograd.grad(e, mu)
        return -self._sum(g)

    def dipole_field(self, pos, cell, pairs, v, pol: Optional[Tensor] = None) -> Tensor:
        """``T v``: field at every site from dipoles ``v`` alone."""
        n = v.shape[0]
        z3 = v.new_zeros(n, 3, 3)
        vv = v.detach().clone().requires_grad_(True)
        with torch.enable_grad():
            e = self.electrostatic(pos.detach(), cell.detach(), pairs, v.new_zeros(n), vv, z3, pol=pol)
            (g,) = torch.autograd.grad(e, vv)
        return -self._sum(g)

    def induce(self, pos, cell, pairs, q, d, Q, pol, mu0: Optional[Tensor] = None, check_every: int = 4):
        """Induced dipoles by Jacobi-preconditioned CG on ``(alpha^-1 - T) mu = F_perm``.

        ``T`` is applied directly (:class:`DipoleOperator`): the real-space pair couplings are
        formed once, the reciprocal part is one spread, FFT and gather of the dipoles. The
        convergence test runs on the device every iteration -- a converged solve freezes (zero
        steps), so the result is the one of stopping there -- and is read back every
        ``check_every`` iterations only."""
        damp = pol if self.thole is not None else None
        F = self.field(pos, cell, pairs, q, d, Q, pol=damp) / KE        # fields in e / A^2 (Coulomb units)
        return self.solve(pos, cell, pairs, F, pol, mu0, check_every)

    def solve(self, pos, cell, pairs, F, pol, mu0: Optional[Tensor] = None, check_every: int = 4):
        """The CG iterations of :meth:`induce` for a given permanent field ``F`` (Coulomb units)."""
        damp = pol if self.thole is not None else None
        inv_a = 1.0 / pol[:, None]
        if self.mutual_intra:              # intramolecular dipole pairs as ordinary damped pairs
            pairs = (pairs[0], pairs[1], pairs[2], torch.zeros_like(pairs[3]))
        T = DipoleOperator(self, pos, cell, pairs, damp)

        def A(v):
            return inv_a * v - T(v)

        mu = pol[:, None] * F if mu0 is None else mu0.detach().clone()
        r = F - A(mu)
        z = pol[:, None] * r
        p_ = z.clone()
        rz = (r * z).sum()
        done = torch.zeros((), dtype=torch.bool, device=pos.device)
        iters = torch.zeros((), dtype=torch.long, device=pos.device)
        err = torch.sqrt(((pol[:, None] * r) ** 2).sum(-1).mean())
        it = 0
        for it in range(1, self.max_iter + 1):
            Ap = A(p_)
            step = torch.where(done, torch.zeros_like(rz), rz / (p_ * Ap).sum())
            mu = mu + step * p_
            r = r - step * Ap
            z = pol[:, None] * r
            err = torch.where(done, err, torch.sqrt(((pol[:, None] * r) ** 2).sum(-1).mean()))
            iters = torch.where(done, iters, torch.full_like(iters, it))
            done = done | (err < self.tol)
            rz_new = (r * z).sum()
            p_ = torch.where(done, p_, z + (rz_new / rz) * p_)
            rz = torch.where(done, rz, rz_new)
            if it % check_every == 0 and bool(done):
                break
        return mu.detach(), int(iters), float(err)

    def forward(self, pos: Tensor, cell: Tensor, q: Tensor, d: Tensor, Q: Tensor, pol: Tensor,
                molecule: Optional[Tensor] = None, compute_forces: bool = True,
                mu0: Optional[Tensor] = None) -> Dict[str, Tensor]:
        pairs = self.pairs(pos, cell, molecule)
        mu, iters, err = self.induce(pos, cell, pairs, q, d, Q, pol, mu0)
        p = pos.detach().requires_grad_(compute_forces)
        with torch.enable_grad():
            e_total = self.polarizable_energy(p, cell, pairs, q, d, Q, pol, mu)
            out = {"energy": self._sum(e_total.detach().reshape(1))[0], "induced_dipoles": mu,
                   "iterations": torch.tensor(iters), "residual_debye": torch.tensor(err / DEBYE)}
            if compute_forces:
                (g,) = torch.autograd.grad(e_total, p)
                out["forces"] = -self._sum(g)
        if self.mesh_backend is not None and hasattr(self.mesh_backend, "check"):
            self.mesh_backend.check()
        return out
