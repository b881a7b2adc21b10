"""One- and two-center integrals of the MNDO-family ``sp`` Hamiltonians.

* Element quantities: the charge separations of the multipoles (dipole ``dd``,
  quadrupole ``qq``, from the Slater exponents and the period) and the additive
  terms ``rho0``/``rho1``/``rho2`` that make each multipole pair reproduce the
  one-center integrals ``Gss``, ``Hsp`` and ``(Gpp - Gp2) / 2`` at zero
  separation (Dewar & Thiel, Theor. Chim. Acta 46, 89 (1977); reference
  ``sqmnn/models/derived.py:177-330``).
* Two-electron integrals: every orbital product on an atom is a sum of point
  charge multipoles (monopole, three dipoles, three linear and two square
  quadrupoles); a local integral is the sum of the charge-charge interactions
  ``q_a q_b / sqrt(r^2 + (rho_a + rho_b)^2)`` over the multipoles of the two
  products, formed in the pair frame (``z`` from A to B) and rotated to the
  molecular frame. ``(p_x p_y | p_x p_y)`` follows from rotational invariance
  about the axis (reference ``sqmnn/models/twocenter.py:1-16``).
* Overlaps of the Slater orbitals, exact, in prolate spheroidal coordinates:
  each product is a polynomial in ``xi`` and ``eta`` integrated against
  ``exp(-p xi - p t eta)`` by the auxiliary integrals ``A_k`` and ``B_k``
  (Mulliken, Rieke, Orloff & Orloff, J. Chem. Phys. 17, 1248 (1949)).

All quantities are float64 tensors, differentiable in the positions and in the
element parameters.
"""
from __future__ import annotations

import math
from functools import lru_cache
from typing import Dict, Tuple

import numpy as np
import torch
from torch import Tensor

#: Bohr radius (Angstrom) and Hartree energy (eV), CODATA 2018: the values the methods were fitted with.
BOHR = 0.529177210903
HARTREE = 27.211386245988
EV_TO_KCAL = 23.060547830619029

# orbital order of an atom: s, p_x, p_y, p_z
S, X, Y, Z = 0, 1, 2, 3

# the point-charge multipoles of one atom: charges (9, 4), unit offsets (9, 4, 3), which separation
# (0 none, 1 dd, 2 2qq, 3 qq), which additive term (0 rho0, 1 rho1, 2 rho2) and the orbital products
# each contributes to (coefficient tables (9, 4, 4))
_SLOTS = [
    ("Q", [(1.0, (0, 0, 0))], 0, 0, [(S, S), (X, X), (Y, Y), (Z, Z)]),
    ("Dx", [(0.5, (1, 0, 0)), (-0.5, (-1, 0, 0))], 1, 1, [(S, X), (X, S)]),
    ("Dy", [(0.5, (0, 1, 0)), (-0.5, (0, -1, 0))], 1, 1, [(S, Y), (Y, S)]),
    ("Dz", [(0.5, (0, 0, 1)), (-0.5, (0, 0, -1))], 1, 1, [(S, Z), (Z, S)]),
    ("Qxx", [(0.25, (1, 0, 0)), (0.25, (-1, 0, 0)), (-0.5, (0, 0, 0))], 2, 2, [(X, X)]),
    ("Qyy", [(0.25, (0, 1, 0)), (0.25, (0, -1, 0)), (-0.5, (0, 0, 0))], 2, 2, [(Y, Y)]),
    ("Qzz", [(0.25, (0, 0, 1)), (0.25, (0, 0, -1)), (-0.5, (0, 0, 0))], 2, 2, [(Z, Z)]),
    ("Qxz", [(0.25, (1, 0, 1)), (0.25, (-1, 0, -1)), (-0.25, (1, 0, -1)), (-0.25, (-1, 0, 1))], 3, 2,
     [(X, Z), (Z, X)]),
    ("Qyz", [(0.25, (0, 1, 1)), (0.25, (0, -1, -1)), (-0.25, (0, 1, -1)), (-0.25, (0, -1, 1))], 3, 2,
     [(Y, Z), (Z, Y)]),
]


@lru_cache(maxsize=None)
def _slot_arrays():
    q = np.zeros((9, 4))
    u = np.zeros((9, 4, 3))
    coef = np.zeros((9, 4, 4))
    for s, (_, charges, _, _, products) in enumerate(_SLOTS):
        for c, (v, off) in enumerate(charges):
            q[s, c] = v
            u[s, c] = off
        for i, j in products:
            coef[s, i, j] = 1.0
    sep = np.array([row[2] for row in _SLOTS])
    rho = np.array([row[3] for row in _SLOTS])
    return q, u, coef, sep, rho


def _slot_tensors(device, dtype):
    q, u, coef, sep, rho = _slot_arrays()
    as_t = lambda a: torch.as_tensor(a, dtype=dtype, device=device)  # noqa: E731
    return as_t(q), as_t(u), as_t(coef), torch.as_tensor(sep, device=device), torch.as_tensor(rho, device=device)


# --------------------------------------------------------------------------------------------------------------
# element quantities


def _newton_root(residual, x0: Tensor, iters: int = 60) -> Tensor:
    """Root of the scalar equations ``residual(x) = 0`` (elementwise) by damped Newton steps on detached values,
    then one differentiable step, so that ``dx/dtheta = -(dr/dtheta) / (dr/dx)`` (implicit function theorem)."""
    x = x0.detach().clone()
    with torch.enable_grad():
        for _ in range(iters):
            xg = x.clone().requires_grad_(True)
            r = residual(xg, detach=True)
            (dr,) = torch.autograd.grad(r.sum(), xg)
            step = r.detach() / dr
            x_new = x - step
            # keep the iterate positive (the additive terms are positive)
            x_new = torch.where(x_new > 0, x_new, 0.5 * x)
            done = bool((x_new - x).abs().max() <= 1e-15 * x.abs().max().clamp(min=1.0))
            x = x_new
            if done:
                break
        xg = x.clone().requires_grad_(True)
        (dr,) = torch.autograd.grad(residual(xg, detach=True).sum(), xg)
    return x - residual(x, detach=False) / dr.detach()


def element_quantities(z: Tensor, table: Dict[str, Tensor], pqn: Tensor, occ_s: Tensor, occ_p: Tensor,
                       has_p: Tensor) -> Dict[str, Tensor]:
    """Derived quantities of the elements ``z`` (one row each) from their parameter columns ``table``.

    Returns ``dd``, ``qq`` (bohr), ``rho`` ``(n, 3)`` (bohr), ``po9`` (core additive term, bohr),
    ``one_center`` ``(n, 4, 4, 4, 4)`` (eV) and ``eisol`` (eV, energy of the isolated atom)."""
    g = table
    dt = g["USS"].dtype
    hp = has_p.to(dt)
    one = torch.ones_like(g["USS"])
    zs = g["ZS"]
    zp = torch.where(has_p, g["ZP"].clamp(min=0.3), one)
    n = pqn.to(dt)
    dd = (2.0 * n + 1.0) * (4.0 * zs * zp) ** (n + 0.5) / (zs + zp) ** (2.0 * n + 2.0) / math.sqrt(3.0)
    qq = torch.sqrt((4.0 * n * n + 6.0 * n + 2.0) / 20.0) / zp
    dd, qq = dd * hp, qq * hp
    gss = g["GSS"]
    am = torch.where(gss > 1e-20, gss / HARTREE, one)
    hsp = torch.where(has_p, g["HSP"].clamp(min=1e-7), one)
    hpp = (0.5 * (g["GPP"] - g["GP2"])).clamp(min=0.1)
    dd_r = torch.where(has_p, dd, one)
    qq_r = torch.where(has_p, qq, one)

    def r_dipole(x, detach):
        d, h = (dd_r.detach(), hsp.detach()) if detach else (dd_r, hsp)
        return 0.5 * x - 0.5 / torch.sqrt(4.0 * d * d + 1.0 / (x * x)) - h / HARTREE

    def r_quad(x, detach):
        qv, h = (qq_r.detach(), hpp.detach()) if detach else (qq_r, hpp)
        return (0.25 * x - 0.5 / torch.sqrt(4.0 * qv * qv + 1.0 / (x * x))
                + 0.25 / torch.sqrt(8.0 * qv * qv + 1.0 / (x * x)) - h / HARTREE)

    ad = _newton_root(r_dipole, (hsp / (HARTREE * dd_r ** 2)) ** (1.0 / 3.0))
    aq = _newton_root(r_quad, (16.0 * hpp / (HARTREE * 48.0 * qq_r ** 4)) ** 0.2)
    ad = torch.where(has_p, ad, am)
    aq = torch.where(has_p, aq, am)
    rho = torch.stack([0.5 / am, 0.5 / ad, 0.5 / aq], -1)
    po9 = torch.where(g["POC"] > 1e-5, g["POC"], rho[:, 0])

    # one-center integrals (mu nu | la si) of the sp shell
    O = g["USS"].new_zeros(z.shape[0], 4, 4, 4, 4)
    O[:, S, S, S, S] = gss
    hpp_raw = 0.5 * (g["GPP"] - g["GP2"])
    for p in (X, Y, Z):
        O[:, S, S, p, p] = g["GSP"] * hp
        O[:, p, p, S, S] = g["GSP"] * hp
        for a, b, c, d in ((S, p, S, p), (S, p, p, S), (p, S, S, p), (p, S, p, S)):
            O[:, a, b, c, d] = g["HSP"] * hp
        O[:, p, p, p, p] = g["GPP"] * hp
        for q in (X, Y, Z):
            if q != p:
                O[:, p, p, q, q] = g["GP2"] * hp
                for a, b, c, d in ((p, q, p, q), (p, q, q, p)):
                    O[:, a, b, c, d] = hpp_raw * hp

    # energy of the isolated atom in its reference configuration
    ios, iop = occ_s.to(dt), occ_p.to(dt)
    ll = torch.minimum(iop, 6.0 - iop)
    eisol = (g["USS"] * ios + g["UPP"] * iop + gss * (ios - 1.0).clamp(min=0.0)
             + g["GPP"] * (-0.25 * ll * (ll - 1.0)) + g["GSP"] * ios * iop
             + g["GP2"] * (0.5 * iop * (iop - 1.0) + 0.25 * ll * (ll - 1.0)) + g["HSP"] * (-0.5 * iop * ios))
    eisol = torch.where(z == 1, g["USS"], eisol)
    return dict(dd=dd, qq=qq, rho=rho, po9=po9, one_center=O, eisol=eisol)


# --------------------------------------------------------------------------------------------------------------
# pair frames


def pair_frames(vec: Tensor) -> Tuple[Tensor, Tensor]:
    """Distances ``r`` and frames ``(n, 3, 3)`` whose rows are the local x, y, z axes (z along ``vec``).

    The results of this module do not depend on the choice of x and y (the local integrals are invariant
    under rotations about z), so any smooth-enough choice serves."""
    r = vec.norm(dim=-1)
    ez = vec / r[:, None]
    helper = torch.zeros_like(ez)
    use_x = ez[:, 0].abs() < 0.9
    helper[:, 0] = use_x.to(vec.dtype)
    helper[:, 1] = (~use_x).to(vec.dtype)
    ex = helper - (helper * ez).sum(-1, keepdim=True) * ez
    ex = ex / ex.norm(dim=-1, keepdim=True)
    ey = torch.cross(ez, ex, dim=-1)
    return r, torch.stack([ex, ey, ez], 1)


def orbital_rotation(frames: Tensor) -> Tensor:
    """``T (n, 4, 4)``: molecular orbital ``i`` = sum_a ``T[i, a]`` local orbital ``a`` (s unchanged)."""
    T = frames.new_zeros(frames.shape[0], 4, 4)
    T[:, 0, 0] = 1.0
    T[:, 1:, 1:] = frames.transpose(1, 2)
    return T


# --------------------------------------------------------------------------------------------------------------
# two-center electron repulsion and core attraction


def _separations(dd: Tensor, qq: Tensor) -> Tensor:
    """Per atom the separation of each multipole slot ``(n, 9)`` (bohr)."""
    _, _, _, sep, _ = _slot_tensors(dd.device, dd.dtype)
    cols = torch.stack([torch.zeros_like(dd), dd, 2.0 * qq, qq], -1)
    return cols[:, sep]


def _slot_rho(rho: Tensor) -> Tensor:
    _, _, _, _, rsel = _slot_tensors(rho.device, rho.dtype)
    return rho[:, rsel]


def local_repulsion(r_bohr: Tensor, dA: Tensor, rhoA: Tensor, dB: Tensor, rhoB: Tensor) -> Tensor:
    """Local-frame integrals ``(n, 4, 4, 4, 4)`` (eV) of pairs at distances ``r_bohr``; ``d*`` ``(n, 9)``
    are the slot separations and ``rho*`` ``(n, 9)`` the slot additive terms of the two atoms."""
    q, u, coef, _, _ = _slot_tensors(r_bohr.device, r_bohr.dtype)
    pa = dA[:, :, None, None] * u                                   # (n, 9, 4, 3)
    pb = dB[:, :, None, None] * u
    pb = pb + torch.stack([torch.zeros_like(r_bohr)] * 2 + [r_bohr], -1)[:, None, None, :]
    diff = pb[:, None, None, :, :, :] - pa[:, :, :, None, None, :]  # (n, 9, 4, 9, 4, 3)
    rr = (rhoA[:, :, None] + rhoB[:, None, :])                      # (n, 9, 9)
    dist2 = (diff * diff).sum(-1) + (rr * rr)[:, :, None, :, None]
    inter = (q[None, :, :, None, None] * q[None, None, None, :, :] * torch.rsqrt(dist2)).sum((2, 4))  # (n, 9, 9)
    W = torch.einsum("sij,tkl,nst->nijkl", coef, coef, inter) * HARTREE
    pxy = 0.5 * (W[:, X, X, X, X] - W[:, X, X, Y, Y])
    W = W.clone()
    for a, b, c, d in ((X, Y, X, Y), (X, Y, Y, X), (Y, X, X, Y), (Y, X, Y, X)):
        W[:, a, b, c, d] = pxy
    return W


def local_core_attraction(r_bohr: Tensor, dA: Tensor, rhoA: Tensor, po9_core: Tensor, sign: float) -> Tensor:
    """Local-frame ``(mu nu | core)`` ``(n, 4, 4)`` (eV, unit core charge) of the electrons of atom A with the
    core of the other atom at ``sign * r`` on the z axis (a monopole with additive term ``po9_core``)."""
    q, u, coef, _, _ = _slot_tensors(r_bohr.device, r_bohr.dtype)
    pa = dA[:, :, None, None] * u
    core = torch.stack([torch.zeros_like(r_bohr)] * 2 + [sign * r_bohr], -1)[:, None, None, :]
    diff = core - pa
    rr = rhoA + po9_core[:, None]
    inter = (q[None] * torch.rsqrt((diff * diff).sum(-1) + (rr * rr)[:, :, None])).sum(-1)   # (n, 9)
    return torch.einsum("sij,ns->nij", coef, inter) * HARTREE


def rotate4(W: Tensor, T: Tensor) -> Tensor:
    """``W'[i,j,k,l] = T[i,a] T[j,b] T[k,c] T[l,d] W[a,b,c,d]`` per pair."""
    W = torch.einsum("nia,nabcd->nibcd", T, W)
    W = torch.einsum("njb,nibcd->nijcd", T, W)
    W = torch.einsum("nkc,nijcd->nijkd", T, W)
    return torch.einsum("nld,nijkd->nijkl", T, W)


def rotate2(V: Tensor, T: Tensor) -> Tensor:
    return torch.einsum("nia,nab,njb->nij", T, V, T)


# --------------------------------------------------------------------------------------------------------------
# overlaps of Slater orbitals


def _pmul(a: Dict, b: Dict) -> Dict:
    out: Dict = {}
    for (i1, j1), c1 in a.items():
        for (i2, j2), c2 in b.items():
            key = (i1 + i2, j1 + j2)
            out[key] = out.get(key, 0.0) + c1 * c2
    return out


def _ppow(a: Dict, k: int) -> Dict:
    out = {(0, 0): 1.0}
    for _ in range(k):
        out = _pmul(out, a)
    return out


@lru_cache(maxsize=None)
def overlap_polynomial(na: int, la: int, nb: int, lb: int, pi: bool) -> Tuple[np.ndarray, float]:
    """Coefficients ``c[k, l]`` of ``xi^k eta^l`` in the spheroidal integrand of the overlap of the Slater
    orbitals ``(na, la)`` on A and ``(nb, lb)`` on B (B on +z; ``pi`` for the p_x-p_x product), and the
    angular prefactor (the ``phi`` integral times the real harmonics' constants)."""
    plus, minus = {(1, 0): 1.0, (0, 1): 1.0}, {(1, 0): 1.0, (0, 1): -1.0}
    vol = {(2, 0): 1.0, (0, 2): -1.0}
    if pi:
        rho2 = _pmul({(2, 0): 1.0, (0, 0): -1.0}, {(0, 0): 1.0, (0, 2): -1.0})
        poly = _pmul(_pmul(_ppow(plus, na - 2), _ppow(minus, nb - 2)), _pmul(rho2, vol))
        pref = 0.75
    else:
        za, zb = {(0, 0): 1.0, (1, 1): 1.0}, {(1, 1): 1.0, (0, 0): -1.0}
        poly = _pmul(_pmul(_ppow(plus, na - 1 - la), _ppow(minus, nb - 1 - lb)),
                     _pmul(_pmul(_ppow(za, la), _ppow(zb, lb)), vol))
        pref = 0.5 * math.sqrt(3.0) ** (la + lb)
    deg = max(max(k, l) for k, l in poly) + 1
    c = np.zeros((deg, deg))
    for (k, l), v in poly.items():
        c[k, l] += v
    return c, pref


def _a_integrals(p: Tensor, kmax: int) -> Tensor:
    """``A_k(p) = int_1^inf x^k exp(-p x) dx`` for k = 0..kmax, ``(n, kmax+1)``."""
    e = torch.exp(-p)
    out = [e / p]
    for k in range(1, kmax + 1):
        out.append((k * out[-1] + e) / p)
    return torch.stack(out, -1)


def _b_integrals(x: Tensor, kmax: int) -> Tensor:
    """``B_k(x) = int_-1^1 y^k exp(-x y) dy`` for k = 0..kmax, ``(n, kmax+1)``: the power series for
    ``|x| <= 6`` and the upward recursion (stable there) above."""
    small = x.abs() <= 6.0
    xs = torch.where(small, x, torch.zeros_like(x))
    xl = torch.where(small, torch.full_like(x, 7.0), x).clamp(-600.0, 600.0)
    ep, em = torch.exp(xl), torch.exp(-xl)
    rec = [(ep - em) / xl]
    for k in range(1, kmax + 1):
        rec.append(((-1.0) ** k * ep - em + k * rec[-1]) / xl)
    rec_t = torch.stack(rec, -1)
    terms = 90
    m = torch.arange(terms, dtype=x.dtype, device=x.device)
    # (-x)^m / m! by a cumulative product (stable for |x| <= 6)
    ratio = torch.cat([torch.ones_like(xs)[:, None], (-xs[:, None]) / m[1:][None, :]], -1)
    powfac = torch.cumprod(ratio, -1)                               # (n, terms)
    ks = torch.arange(kmax + 1, device=x.device)
    km = ks[:, None] + torch.arange(terms, device=x.device)[None, :]  # (K, terms)
    w = torch.where(km % 2 == 0, 2.0 / (km + 1).to(x.dtype), torch.zeros_like(km, dtype=x.dtype))
    ser = (powfac[:, None, :] * w[None]).sum(-1)
    return torch.where(small[:, None], ser, rec_t)


def _normalization(n: int, zeta: Tensor) -> Tensor:
    return (2.0 * zeta) ** (n + 0.5) / math.sqrt(math.factorial(2 * n))


def sto_overlap(na: int, la: int, za: Tensor, nb: int, lb: int, zb: Tensor, r_bohr: Tensor, pi: bool = False) -> Tensor:
    """Overlap of Slater orbitals ``(na, la, za)`` on A and ``(nb, lb, zb)`` on B, with B at ``r_bohr`` on the z axis
    of A (``la``/``lb`` 1 with ``pi`` False: p_z; with ``pi``: the p_x-p_x overlap)."""
    c, pref = overlap_polynomial(na, la, nb, lb, pi)
    kmax = c.shape[0] - 1
    p = 0.5 * r_bohr * (za + zb)
    pt = 0.5 * r_bohr * (za - zb)
    A = _a_integrals(p, kmax)
    Bt = _b_integrals(pt, kmax)
    ct = torch.as_tensor(c, dtype=r_bohr.dtype, device=r_bohr.device)
    s = torch.einsum("nk,kl,nl->n", A, ct, Bt)
    return pref * _normalization(na, za) * _normalization(nb, zb) * (0.5 * r_bohr) ** (na + nb + 1) * s


def local_overlaps(n_a: int, n_b: int, zs_a: Tensor, zp_a: Tensor, zs_b: Tensor, zp_b: Tensor, r_bohr: Tensor,
                   p_a: bool, p_b: bool) -> Tensor:
    """Local-frame overlap blocks ``(n, 4, 4)`` of pairs whose atoms have principal quantum numbers ``n_a``,
    ``n_b`` (the same for the s and p shells of an sp atom); ``p_*`` whether the atom has p orbitals."""
    out = r_bohr.new_zeros(r_bohr.shape[0], 4, 4)
    out[:, S, S] = sto_overlap(n_a, 0, zs_a, n_b, 0, zs_b, r_bohr)
    if p_b:
        out[:, S, Z] = sto_overlap(n_a, 0, zs_a, n_b, 1, zp_b, r_bohr)
    if p_a:
        out[:, Z, S] = sto_overlap(n_a, 1, zp_a, n_b, 0, zs_b, r_bohr)
    if p_a and p_b:
        out[:, Z, Z] = sto_overlap(n_a, 1, zp_a, n_b, 1, zp_b, r_bohr)
        pp = sto_overlap(n_a, 1, zp_a, n_b, 1, zp_b, r_bohr, pi=True)
        out[:, X, X] = pp
        out[:, Y, Y] = pp
    return out
