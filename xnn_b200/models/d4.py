"""Grimme D4 dispersion: EEQ partial charges, charge-scaled dynamic polarizabilities, C6 by
Casimir-Polder integration, BJ-damped two-body and ATM three-body energies.

Written from Caldeweyher et al., J. Chem. Phys. 150, 154122 (2019), with the conventions of the
reference's ``src/xnn/common/models/d4.py`` (``DFTD4`` at ``:266``) so the numbers agree: the
error-function coordination number (k0 = 7.5, 4/3-scaled covalent radii) weighted by the
electronegativity factor (k1..k3), the softly capped EEQ coordination number, the EEQ solve with
the Gaussian-charge Coulomb matrix and the total-charge constraint, the N^s Gaussian weights
(beta2 = 6) with the highest-CN fallback, the charge scaling zeta of the reference
polarizabilities (ga = 3, gc = 2), the 23-point Casimir-Polder trapezoid grid, and the ATM term
from neutral (q = 0) polarizabilities. Reference data: the published D4 tables
(``d4_reference.npz``, see :mod:`xnn_b200.models.dispersion`).

Built: the dense regime for isolated and periodic structures (the periodic EEQ Coulomb matrix from
Wigner-Seitz images and Ewald sums with the dftd4 splitting rule). Not built: the large-system
iterative EEQ and the lattice tail correction.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np
import torch
from torch import Tensor, nn

from ..ops.scatter import scatter_sum, structure_sum
from .dispersion import (BOHR, HARTREE, DispersionCorrection, atm_kernel_ok, evaluate_on_graph,
                         gaussian_reference_weights, load_tables, options_from_extra, switching_function,
                         three_body_energy, three_body_energy_factored)
from .registry import register_model

KCN, K4, K5, K6 = 7.5, 4.10451, 19.08857, 2.0 * 11.28174 ** 2
EEQ_CN_MAX, EEQ_CN_REG = 8.0, 1.0e-14
MAX_Z = 103
CUTOFF_PAIR_AU, CUTOFF_TRIPLE_AU, CUTOFF_CN_AU, CUTOFF_EEQ_CN_AU = 60.0, 40.0, 30.0, 25.0
FREQ = [0.000001, 0.05, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0, 1.2, 1.4, 1.6, 1.8, 2.0, 2.5, 3.0, 4.0,
        5.0, 7.5, 10.0]
CP_WEIGHTS = [0.5 * ((FREQ[k] - FREQ[k - 1] if k > 0 else 0.0) + (FREQ[k + 1] - FREQ[k] if k < len(FREQ) - 1 else 0.0))
              for k in range(len(FREQ))]


WS_TOL = 0.01          # bohr^2: images within this of the nearest count as equivalent
EWALD_REP = 2          # +-2 real and reciprocal lattice windows of the periodic EEQ


def _ewald_balance(alpha: float, rlen: float, dlen: float, vol: float) -> float:
    rec = lambda g: 4.0 * math.pi * math.exp(-0.25 * g * g / (alpha * alpha)) / (vol * g * g)  # noqa: E731
    direct = lambda r: math.erfc(alpha * r) / r  # noqa: E731
    return (rec(4.0 * rlen) - rec(5.0 * rlen)) - (direct(2.0 * dlen) - direct(3.0 * dlen))


def ewald_alpha(rlen: float, dlen: float, vol: float) -> float:
    """The Ewald splitting parameter of the periodic EEQ (the dftd4 rule): the ``alpha`` at which the
    last real-space and reciprocal-space shells of the +-2 windows carry equal weight, bracketed by
    doubling from 1e-8 and bisected to sqrt(float32 eps); 0.25 when no bracket is found."""
    tol = 1.4901161193847656e-08
    alpha = 1.0e-8
    d = _ewald_balance(alpha, rlen, dlen, vol)
    n = 0
    while d < -tol and n < 2000:
        alpha *= 2.0
        d = _ewald_balance(alpha, rlen, dlen, vol)
        n += 1
    if n == 0 or n >= 2000:
        return 0.25
    left, n = 0.5 * alpha, 0
    while d < tol and n < 2000:
        alpha *= 2.0
        d = _ewald_balance(alpha, rlen, dlen, vol)
        n += 1
    if n >= 2000:
        return 0.25
    right = alpha
    alpha = 0.5 * (left + right)
    d, n = _ewald_balance(alpha, rlen, dlen, vol), 0
    while abs(d) > tol and n <= 30:
        left, right = (alpha, right) if d < 0.0 else (left, alpha)
        alpha = 0.5 * (left + right)
        d = _ewald_balance(alpha, rlen, dlen, vol)
        n += 1
    return 0.25 if n > 30 else alpha


def _zeta(a: float, c, qref, qmod):
    """Charge scaling exp(a (1 - exp(c (1 - qref / qmod)))), exp(a) for negative qmod."""
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        s = np.exp(a * (1.0 - np.exp(c * (1.0 - qref / qmod))))
    return np.where(qmod < 0.0, np.exp(a), s)


def _matrix_free_ok(pos: Tensor) -> bool:
    if not (pos.is_cuda and pos.dtype == torch.float64):
        return False
    from .. import _ext
    return _ext.cuda_available() and hasattr(_ext.ops(), "coulomb_matvec")


def _cg2(apply, rhs: Tensor, diag: Tensor, tol: float, max_iter: int) -> Tensor:
    """Jacobi-preconditioned conjugate gradients on the columns of ``rhs (n, k)`` together."""
    x = rhs / diag[:, None]
    r = rhs - apply(x)
    z = r / diag[:, None]
    p = z.clone()
    rz = (r * z).sum(0)
    bnorm = rhs.norm(dim=0).clamp_min(1e-300)
    for _ in range(max_iter):
        Ap = apply(p)
        alpha = rz / (p * Ap).sum(0)
        x = x + alpha * p
        r = r - alpha * Ap
        if bool(((r.norm(dim=0) / bnorm) < tol).all()):
            break
        z = r / diag[:, None]
        rz_new = (r * z).sum(0)
        p = z + (rz_new / rz) * p
        rz = rz_new
    return x


class _EEQMatrixFree(torch.autograd.Function):
    """EEQ charges of a molecule from ``A q = x - lambda 1``, ``sum q = Q`` (``A`` the erf-screened
    Coulomb matrix plus the diagonal hardness) without forming ``A``: the product is the all-pairs
    kernel ``coulomb_matvec``; the two solves ``A s = x`` and ``A u = 1`` run together and
    ``q = s - (sum s - Q) / sum u * u``. The backward pass solves the adjoint the same way and
    differentiates the matrix through ``coulomb_bilinear_grad`` (implicit differentiation)."""

    @staticmethod
    def forward(ctx, pos, x, rad, diag, Q, tol, max_iter):
        from .. import _ext
        C = _ext.ops()
        posc = pos.detach().contiguous()

        def apply(v):
            return C.coulomb_matvec(posc, rad, v.contiguous()) + diag[:, None] * v
        rhs = torch.stack([x.detach(), torch.ones_like(x)], 1)
        su = _cg2(apply, rhs, diag, tol, max_iter)
        s, u = su[:, 0], su[:, 1]
        q = s - ((s.sum() - Q) / u.sum()) * u
        ctx.save_for_backward(posc, rad, diag, q, u)
        ctx.tol, ctx.max_iter = tol, max_iter
        return q

    @staticmethod
    def backward(ctx, g):
        from .. import _ext
        C = _ext.ops()
        posc, rad, diag, q, u = ctx.saved_tensors

        def apply(v):
            return C.coulomb_matvec(posc, rad, v.contiguous()) + diag[:, None] * v
        sg = _cg2(apply, g.contiguous()[:, None], diag, ctx.tol, ctx.max_iter)[:, 0]
        mu = sg - (sg.sum() / u.sum()) * u                     # the constrained adjoint (sum mu = 0)
        g_pos = -C.coulomb_bilinear_grad(posc, rad, mu.contiguous(), q.contiguous())
        return g_pos, mu, None, None, None, None, None


class DFTD4(nn.Module):
    def __init__(self, s6: float = 1.0, s8: float = 1.20065498, a1: float = 0.40085597, a2: float = 5.02928789,
                 s9: float = 1.0, alp: float = 16.0, ga: float = 3.0, gc: float = 2.0, wf: float = 6.0,
                 cutoff_pair: float = CUTOFF_PAIR_AU * BOHR, cutoff_triple: float = CUTOFF_TRIPLE_AU * BOHR,
                 cutoff_cn: float = CUTOFF_CN_AU * BOHR, cutoff_eeq_cn: float = CUTOFF_EEQ_CN_AU * BOHR,
                 switch_width_pair: float = 0.0, switch_width_triple: float = 0.0, trainable: bool = False,
                 reference_charges: str = "eeq", **unused):
        super().__init__()
        self.ga, self.gc, self.wf, self.alp = float(ga), float(gc), float(wf), float(alp)
        self.cutoff_pair, self.cutoff_triple = float(cutoff_pair), float(cutoff_triple)
        self.cutoff_cn, self.cutoff_eeq_cn = float(cutoff_cn), float(cutoff_eeq_cn)
        self.cutoff = max(self.cutoff_pair, self.cutoff_triple, self.cutoff_cn, self.cutoff_eeq_cn)
        self.switch_width_pair, self.switch_width_triple = float(switch_width_pair), float(switch_width_triple)
        self.n_features = 3
        #: the three-body term on the CUDA kernel (float64 CUDA inputs); False: the tensor formulas
        self.use_kernels = True
        #: molecules with more atoms solve EEQ without forming the matrix (CUDA float64), to this
        #: relative residual
        self.eeq_dense_max, self.eeq_tol, self.eeq_max_iter = 2000, 1e-12, 500
        dt = torch.get_default_dtype()
        for name, v in [("s6", s6), ("s8", s8), ("a1", a1), ("a2", a2), ("s9", s9)]:
            t = torch.tensor(float(v), dtype=dt)
            if trainable:
                setattr(self, name, nn.Parameter(t))
            else:
                self.register_buffer(name, t)
        ref = load_tables("d4_reference.npz")
        if reference_charges not in ("eeq", "gfn2"):
            raise ValueError("reference_charges must be 'eeq' or 'gfn2'")
        if reference_charges == "gfn2":
            ref = dict(ref, refq=ref["refq_gfn2"], refh=ref["refh_gfn2"])
        buf = lambda n, a, d=dt: self.register_buffer(n, torch.tensor(a, dtype=d), persistent=False)  # noqa: E731
        buf("rcov", 4.0 / 3.0 * ref["covalent_radius_aa"] / BOHR)
        buf("en", ref["pauling_en"])
        buf("zeff", ref["zeff"])
        buf("hardness", ref["hardness"])
        zz = np.arange(ref["r4r2_raw"].shape[0], dtype=np.float64)
        buf("r4r2", np.sqrt(0.5 * ref["r4r2_raw"] * np.sqrt(zz)))
        for k in ("eeq_chi", "eeq_eta", "eeq_kcnchi", "eeq_rad"):
            buf(k, np.nan_to_num(ref[k], nan=0.0))
        buf("nref", ref["nref"], torch.long)
        buf("ngw", ref["ngw"], torch.long)
        self.max_ngw = int(ref["ngw"].max())
        buf("refcn", ref["refcn"])
        buf("refq", ref["refq"])
        buf("refalpha", self._reference_polarizabilities(ref))
        buf("cp_weights", CP_WEIGHTS)

    def _reference_polarizabilities(self, ref) -> np.ndarray:
        """``alpha_A,ref(i w)`` (23, 7, Z): the reference molecule's TD-DFT polarizability minus
        its charge-scaled secondary systems, times the reference's scale, clamped at zero."""
        sys = ref["refsys"]
        present = sys > 0
        idx = np.where(present, sys, 0)
        zx = ref["zeff"][idx]
        hx = ref["hardness"][idx] * self.gc
        scale = _zeta(self.ga, hx, zx, ref["refh"] + zx)
        aiw_x = ref["sscale"][idx] * ref["secaiw"][:, idx] * scale
        alpha = ref["ascale"] * (ref["alphaiw"] - ref["hcount"] * aiw_x)
        return np.where(present, np.maximum(alpha, 0.0), 0.0)

    # ------------------------------------------------------------------ pieces (atomic units)
    def coordination_numbers(self, z, edge_index, r, n):
        src, dst = edge_index[0], edge_index[1]
        zi, zj = z[dst], z[src]
        rc = self.rcov[zi] + self.rcov[zj]
        count = 0.5 * (1.0 + torch.erf(-KCN * (r - rc) / rc))
        enf = K4 * torch.exp(-((self.en[zi] - self.en[zj]).abs() + K5) ** 2 / K6)
        cn_d4 = scatter_sum(torch.where(r <= self.cutoff_cn / BOHR, enf * count, torch.zeros_like(count)), dst, n)
        raw = scatter_sum(torch.where(r <= self.cutoff_eeq_cn / BOHR, count, torch.zeros_like(count)), dst, n)
        cn_eeq = math.log(1.0 + math.exp(EEQ_CN_MAX)) - torch.log(1.0 + torch.exp(EEQ_CN_MAX - raw))
        return cn_d4, cn_eeq

    def coulomb_matrix_periodic(self, z: Tensor, pos: Tensor, cell: Tensor) -> Tensor:
        """The EEQ Coulomb matrix of a periodic structure (bohr): for every pair the Wigner-Seitz
        images (the nearest of the 27 neighbouring cells, ties within ``WS_TOL`` shared equally),
        each an Ewald sum of the Gaussian-charge kernel over +-2 real and reciprocal windows; the
        diagonal carries the hardness, the self term and the ``-2 alpha / sqrt(pi)`` correction."""
        n, dev, dt = pos.shape[0], pos.device, pos.dtype
        vol = torch.linalg.det(cell).abs()
        recip = 2.0 * math.pi * torch.linalg.inv(cell).t()
        alpha = ewald_alpha(float(torch.linalg.norm(recip, dim=1).min()), float(torch.linalg.norm(cell, dim=1).min()),
                            float(vol))
        one = torch.arange(-1, 2, device=dev)
        t27 = torch.cartesian_prod(one, one, one).to(dt) @ cell
        two = torch.arange(-EWALD_REP, EWALD_REP + 1, device=dev)
        grid = torch.cartesian_prod(two, two, two)
        t125 = grid.to(dt) @ cell
        g = grid[(grid != 0).any(1)].to(dt) @ recip
        g2 = (g * g).sum(-1)
        g_fac = 4.0 * math.pi / vol * torch.exp(-0.25 * g2 / (alpha * alpha)) / g2
        rad2 = self.eeq_rad[z] ** 2
        gamma = torch.rsqrt(rad2[:, None] + rad2[None, :])
        d = pos[None, :, :] - pos[:, None, :]
        d = d - torch.round(d.detach() @ torch.linalg.inv(cell.detach())) @ cell
        d_img = d[:, :, None, :] + t27[None, None]
        r2 = (d_img * d_img).sum(-1)
        thr = 1.4901161193847656e-08
        r2 = torch.where(r2 < thr, torch.full_like(r2, math.inf), r2)
        sel = (r2 - r2.min(-1, keepdim=True).values) <= WS_TOL
        n_img = sel.sum(-1).to(dt)
        ii, jj, kk = torch.nonzero(sel).unbind(1)
        vec = d_img[ii, jj, kk]
        vt = vec[:, None, :] + t125[None]
        r2t = (vt * vt).sum(-1)
        keep = r2t >= thr * thr
        rs = torch.sqrt(torch.where(keep, r2t, torch.ones_like(r2t)))
        kern = (torch.erf(gamma[ii, jj][:, None] * rs) - torch.erf(alpha * rs)) / rs
        a_dir = torch.where(keep, kern, torch.zeros_like(kern)).sum(-1)
        a_rec = (torch.cos(vec @ g.t()) * g_fac[None]).sum(-1)
        A = scatter_sum((a_dir + a_rec) / n_img[ii, jj], ii * n + jj, n * n).view(n, n)
        return A + torch.diag(self.eeq_eta[z] + math.sqrt(2.0 / math.pi) / self.eeq_rad[z]
                              - 2.0 * alpha / math.sqrt(math.pi))

    def eeq_charges(self, z, pos, cn_eeq, total_charge, cell: Optional[Tensor] = None) -> Tensor:
        """EEQ charges of one structure (positions and cell in bohr); ``cell`` for a periodic one.
        Molecules above :attr:`eeq_dense_max` atoms on a CUDA float64 device take the matrix-free
        solve (:class:`_EEQMatrixFree`)."""
        n = pos.shape[0]
        if cell is None and n > self.eeq_dense_max and _matrix_free_ok(pos):
            x = -self.eeq_chi[z] + self.eeq_kcnchi[z] * cn_eeq / torch.sqrt(cn_eeq + EEQ_CN_REG)
            rad = self.eeq_rad[z].contiguous()
            diag = (self.eeq_eta[z] + math.sqrt(2.0 / math.pi) / self.eeq_rad[z]).contiguous()
            return _EEQMatrixFree.apply(pos, x, rad, diag, float(total_charge), self.eeq_tol, self.eeq_max_iter)
        if cell is not None:
            A = self.coulomb_matrix_periodic(z, pos, cell)
        else:
            rad2 = self.eeq_rad[z] ** 2
            gamma = torch.rsqrt(rad2[:, None] + rad2[None, :])
            eye = torch.eye(n, dtype=torch.bool, device=pos.device)
            dvec = pos[None, :, :] - pos[:, None, :]
            r2 = (dvec * dvec).sum(-1)
            r = torch.sqrt(torch.where(eye, torch.ones_like(r2), r2))
            A = torch.where(eye, torch.zeros_like(r), torch.erf(gamma * r) / r)
            A = A + torch.diag(self.eeq_eta[z] + math.sqrt(2.0 / math.pi) / self.eeq_rad[z])
        x = -self.eeq_chi[z] + self.eeq_kcnchi[z] * cn_eeq / torch.sqrt(cn_eeq + EEQ_CN_REG)
        ones = torch.ones((n, 1), dtype=pos.dtype, device=pos.device)
        zero = torch.zeros((1, 1), dtype=pos.dtype, device=pos.device)
        full = torch.cat([torch.cat([A, ones], 1), torch.cat([ones.t(), zero], 1)], 0)
        rhs = torch.cat([x, torch.as_tensor(total_charge).reshape(1).to(device=pos.device, dtype=pos.dtype)])[:, None]
        return torch.linalg.solve(full, rhs)[:n, 0]

    def gaussian_weights(self, z, cn):
        refcn = self.refcn[:, z].t()
        ngw = self.ngw[:, z].t()
        valid = torch.arange(refcn.shape[1], device=z.device)[None, :] < self.nref[z][:, None]
        eps = 1.0842021724855044e-19 if cn.dtype == torch.float32 else 1.4916681462400413e-154
        return gaussian_reference_weights(cn, refcn, valid, self.wf, ngw, eps)

    def charge_scaling(self, z, q):
        zi = self.zeff[z][:, None]
        gi = (self.hardness[z] * self.gc)[:, None]
        qmod = q[:, None] + zi
        qref = self.refq[:, z].t() + zi
        neg = qmod < 0.0
        safe = torch.where(neg, torch.ones_like(qmod), qmod)
        s = torch.exp(self.ga * (1.0 - torch.exp(gi * (1.0 - qref / safe))))
        return torch.where(neg, torch.full_like(qmod, math.exp(self.ga)), s)

    def dynamic_polarizabilities(self, z, weights):
        return torch.einsum("nr,krn->nk", weights, self.refalpha[:, :, z])

    def two_body_energy(self, z, edge_index, r, alpha_iw, n):
        src, dst = edge_index[0], edge_index[1]
        c6 = (3.0 / math.pi) * (alpha_iw[dst] * alpha_iw[src] * self.cp_weights).sum(-1)
        zi, zj = z[dst], z[src]
        rr = 3.0 * self.r4r2[zi] * self.r4r2[zj]
        r0 = self.a1 * torch.sqrt(rr) + self.a2
        r2 = r * r
        t6 = 1.0 / (r2 ** 3 + r0 ** 6)
        t8 = 1.0 / (r2 ** 4 + r0 ** 8)
        sw = switching_function(r, self.cutoff_pair / BOHR, self.switch_width_pair / BOHR)
        return scatter_sum(-0.5 * c6 * sw * (self.s6 * t6 + self.s8 * rr * t8), dst, n)

    def pair_radius_table(self) -> Tensor:
        return self.a1 * torch.sqrt(3.0 * self.r4r2[:, None] * self.r4r2[None, :]) + self.a2

    # ------------------------------------------------------------------ evaluation
    def evaluate(self, atomic_numbers: Tensor, pos: Tensor, edge_index: Tensor, edge_vec: Tensor, batch: Tensor,
                 num_graphs: int, cell: Tensor, pbc: Tensor, total_charge: Tensor) -> Dict[str, Tensor]:
        z = atomic_numbers
        n = z.shape[0]
        if bool((z > MAX_Z).any()) or bool((z < 1).any()):
            raise ValueError("D4 with EEQ charges supports atomic numbers 1..103")
        periodic = (pbc.any(-1) & (cell.abs().sum((-1, -2)) > 1e-8)).tolist()
        pos_au = pos / BOHR
        vec = edge_vec / BOHR
        r = torch.linalg.norm(vec, dim=-1)
        cn_d4, cn_eeq = self.coordination_numbers(z, edge_index, r, n)
        q = torch.zeros_like(cn_d4)
        for b in range(num_graphs):
            m = torch.nonzero(batch == b).squeeze(1)
            q = q.index_put((m,), self.eeq_charges(z[m], pos_au[m], cn_eeq[m], total_charge[b],
                                                   cell[b] / BOHR if periodic[b] else None))
        alpha_iw = self.dynamic_polarizabilities(z, self.gaussian_weights(z, cn_d4) * self.charge_scaling(z, q))
        in_pair = r <= self.cutoff_pair / BOHR
        e2 = self.two_body_energy(z, edge_index[:, in_pair], r[in_pair], alpha_iw, n)
        e3 = torch.zeros_like(e2)
        if bool(self.s9 != 0.0):
            w0 = self.gaussian_weights(z, cn_d4) * self.charge_scaling(z, torch.zeros_like(q))
            a0 = self.dynamic_polarizabilities(z, w0)
            m3 = r <= self.cutoff_triple / BOHR
            if atm_kernel_ok(vec) and self.use_kernels:
                # C6 factors per atom (no n x n matrix): C6_ij = (3/pi) sum_w cp_w a_i(w) a_j(w)
                e3 = three_body_energy_factored(z, edge_index[:, m3], vec[m3], (3.0 / math.pi) * a0 * self.cp_weights,
                                                a0, self.pair_radius_table(), float(self.s9), self.alp / 3.0,
                                                self.cutoff_triple / BOHR, self.switch_width_triple / BOHR, batch)
            else:
                c6_0 = (3.0 / math.pi) * (a0 * self.cp_weights) @ a0.t()
                e3 = three_body_energy(z, edge_index[:, m3], vec[m3], r[m3], c6_0, self.pair_radius_table(), self.s9,
                                       self.alp / 3.0, self.cutoff_triple / BOHR, self.switch_width_triple / BOHR, n)
        return {"node_energy": (e2 + e3) * HARTREE,
                "energy_2body": structure_sum(e2, batch, num_graphs) * HARTREE,
                "energy_3body": structure_sum(e3, batch, num_graphs) * HARTREE,
                "coordination_numbers": cn_d4, "charges": q, "polarizabilities": alpha_iw[:, 0],
                "dynamic_polarizabilities": alpha_iw,
                "node_features": torch.stack([cn_d4, q, alpha_iw[:, 0]], 1)}

    def forward(self, data) -> Dict[str, Tensor]:
        return evaluate_on_graph(self, data)


D4_KEYS = ("s6", "s8", "a1", "a2", "s9", "alp", "ga", "gc", "wf", "cutoff_pair", "cutoff_triple", "cutoff_cn",
           "cutoff_eeq_cn", "switch_width_pair", "switch_width_triple", "trainable", "reference_charges")


@register_model("d4")
class D4Dispersion(DispersionCorrection):
    """D4 as a potential: standalone, or added to ``model`` (``model.extra["dispersion"]``)."""

    def __init__(self, model=None, **d4_options):
        super().__init__(DFTD4(**{k: v for k, v in d4_options.items() if k in D4_KEYS}), model)

    @property
    def d4(self) -> DFTD4:
        return self.term

    @classmethod
    def from_config(cls, cfg) -> "D4Dispersion":
        return cls(**options_from_extra(dict(getattr(cfg, "extra", {}) or {}), D4_KEYS))
