"""SpookyNet (Unke et al., Nat. Commun. 12, 7273 (2021)): charge and spin embeddings, s/p/d-like
local messages, FAVOR+ self-attention over each structure, and a physical energy split (ZBL-like
repulsion, damped Coulomb, charge-dependent two-body D4).

Behaviour, options and parameter names follow the reference
(``src/xnn/hybnn/models/spookynet.py``: descriptors ``:144``, switch ``:185``, random features
``:201``, residual blocks ``:421,458``, embeddings ``:552,573``, local and nonlocal interactions
``:613,677``, ZBL ``:847``, electrostatics ``:880``, D4 ``:933``, model ``:1060``, checkpoint
renames ``:1634``) so state dicts transplant between the two.

Batched evaluation of the residual MLPs that read the same input (the c/s/p/d and q/k/v networks)
runs them as one stacked product per layer (``baddbmm`` over the stack), a third of the launches
of running them one by one.
"""
from __future__ import annotations

import math
import re
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.radial import ExponentialBernsteinRBF
from ..ops.scatter import gather_rows, scatter_sum
from .base import InteratomicPotential
from .d4 import K4, K5, K6, KCN, CP_WEIGHTS
from .dimenet import glorot_orthogonal_
from .dispersion import BOHR, HARTREE, gaussian_reference_weights, load_tables
from .electrostatics import COULOMB_CONSTANT, all_pairs, coulomb_ewald, ewald_parameters
from .physnet import softplus_inverse
from .registry import register_model

MAX_Z = 87
_SHELLS = ("1s", "2s", "2p", "3s", "3p", "4s", "3d", "4p", "5s", "4d", "5p", "6s", "4f", "5d", "6p")
_HOLD = {"s": 2, "p": 6, "d": 10, "f": 14}
# neutral ground states that leave the aufbau (Madelung) order
_AUFBAU_EXCEPTIONS = {
    24: {"4s": 1, "3d": 5}, 29: {"4s": 1, "3d": 10}, 41: {"5s": 1, "4d": 4}, 42: {"5s": 1, "4d": 5},
    44: {"5s": 1, "4d": 7}, 45: {"5s": 1, "4d": 8}, 46: {"5s": 0, "4d": 10}, 47: {"5s": 1, "4d": 10},
    57: {"4f": 0, "5d": 1}, 58: {"4f": 1, "5d": 1}, 64: {"4f": 7, "5d": 1}, 78: {"6s": 1, "5d": 9},
    79: {"6s": 1, "5d": 10},
}
_NOBLE = (2, 10, 18, 36, 54, 86)


def electron_configurations(max_z: int = MAX_Z - 1) -> np.ndarray:
    """``(max_z + 1, 20)`` element descriptors: Z, the 15 subshell occupations (1s ... 6p) of the
    neutral ground state and the valence occupations (ns, np, (n-1)d, (n-2)f of period n), each
    column scaled to a largest value of one; row 0 is zero."""
    if max_z > 86:
        raise ValueError(f"the descriptor covers Z <= 86, got max_z={max_z}")
    out = np.zeros((max_z + 1, 20))
    for z in range(1, max_z + 1):
        occ, rest = {}, z
        for sh in _SHELLS:
            occ[sh] = min(rest, _HOLD[sh[-1]])
            rest -= occ[sh]
        occ.update(_AUFBAU_EXCEPTIONS.get(z, {}))
        period = 1 + sum(z > e for e in _NOBLE)
        out[z, 0] = z
        out[z, 1:16] = [occ[sh] for sh in _SHELLS]
        out[z, 16:] = [occ.get(f"{period}s", 0), occ.get(f"{period}p", 0), occ.get(f"{period - 1}d", 0),
                       occ.get(f"{period - 2}f", 0)]
    return out / out.max(axis=0)


def smooth_switch(r: Tensor, r_on: float, r_off: float) -> Tensor:
    """1 below ``r_on``, 0 above ``r_off``, ``s(1-x) / (s(1-x) + s(x))`` between with
    ``s(t) = exp(-1/t)`` (t > 0): smooth to every order. Finite gradients everywhere."""
    x = (r - r_on) / (r_off - r_on)
    y = 1.0 - x
    sx = torch.where(x > 0, torch.exp(-1.0 / torch.where(x > 0, x, 1.0)), 0.0)
    sy = torch.where(y > 0, torch.exp(-1.0 / torch.where(y > 0, y, 1.0)), 0.0)
    return torch.where(x <= 0, 1.0, torch.where(x >= 1, 0.0, sy / (sx + sy)))


def orthogonal_random_features(n_features: int, dim: int, generator: Optional[torch.Generator] = None) -> Tensor:
    """``(dim, n_features)`` FAVOR+ projections (Choromanski et al. 2021): blocks of ``dim``
    orthonormal rows (QR of Gaussian matrices), each row rescaled to the norm of an independent
    Gaussian vector."""
    rows = []
    for start in range(0, n_features, dim):
        q, _ = torch.linalg.qr(torch.randn(dim, dim, generator=generator, dtype=torch.float64))
        rows.append(q.t()[:min(dim, n_features - start)])
    norms = torch.randn(n_features, dim, generator=generator, dtype=torch.float64).norm(dim=1, keepdim=True)
    return (norms * torch.cat(rows)).t().contiguous()


class Swish(nn.Module):
    """``alpha x sigmoid(beta x)`` with per-feature ``alpha`` (1) and ``beta`` (1.702)."""

    def __init__(self, n_features: int, alpha: float = 1.0, beta: float = 1.702):
        super().__init__()
        self.alpha = nn.Parameter(torch.full((n_features,), float(alpha)))
        self.beta = nn.Parameter(torch.full((n_features,), float(beta)))

    def forward(self, x: Tensor) -> Tensor:
        return self.alpha * x * torch.sigmoid(self.beta * x)


class ResidualBlock(nn.Module):
    """``x + W2 swish(W1 swish(x))``, ``W2`` zero at start."""

    def __init__(self, n_features: int, bias: bool = True):
        super().__init__()
        self.activation1 = Swish(n_features)
        self.linear1 = nn.Linear(n_features, n_features, bias=bias)
        self.activation2 = Swish(n_features)
        self.linear2 = nn.Linear(n_features, n_features, bias=bias)
        glorot_orthogonal_(self.linear1.weight)
        nn.init.zeros_(self.linear2.weight)
        if bias:
            nn.init.zeros_(self.linear1.bias)
            nn.init.zeros_(self.linear2.bias)

    def forward(self, x: Tensor) -> Tensor:
        return x + self.linear2(self.activation2(self.linear1(self.activation1(x))))


class ResidualMLP(nn.Module):
    """``linear(swish(residual^n(x)))``."""

    def __init__(self, n_features: int, n_residual: int = 1, bias: bool = True, zero_init: bool = False):
        super().__init__()
        self.residual = nn.ModuleList(ResidualBlock(n_features, bias) for _ in range(n_residual))
        self.activation = Swish(n_features)
        self.linear = nn.Linear(n_features, n_features, bias=bias)
        if zero_init:
            nn.init.zeros_(self.linear.weight)
        else:
            glorot_orthogonal_(self.linear.weight)
        if bias:
            nn.init.zeros_(self.linear.bias)

    def forward(self, x: Tensor) -> Tensor:
        for block in self.residual:
            x = block(x)
        return self.linear(self.activation(x))


def _stackable(mlps: List[ResidualMLP]) -> bool:
    first = mlps[0]
    for m in mlps:
        if type(m) is not ResidualMLP or len(m.residual) != len(first.residual):
            return False
        lins = [m.linear] + [b.linear1 for b in m.residual] + [b.linear2 for b in m.residual]
        acts = [m.activation] + [b.activation1 for b in m.residual] + [b.activation2 for b in m.residual]
        if any(type(l) is not nn.Linear or (l.bias is None) != (first.linear.bias is None) for l in lins):
            return False
        if any(type(a) is not Swish for a in acts):
            return False
    return True


def residual_mlps(x: Tensor, mlps: List[ResidualMLP]) -> List[Tensor]:
    """``[m(x) for m in mlps]``: one stacked product per layer when the networks share a shape."""
    if len(mlps) == 1 or not _stackable(mlps):
        return [m(x) for m in mlps]

    def act(h, acts):
        a = torch.stack([s.alpha for s in acts]).unsqueeze(1)
        b = torch.stack([s.beta for s in acts]).unsqueeze(1)
        return a * h * torch.sigmoid(b * h)

    def lin(h, lins):
        w = torch.stack([l.weight for l in lins]).transpose(1, 2)
        if lins[0].bias is None:
            return torch.bmm(h, w)
        return torch.baddbmm(torch.stack([l.bias for l in lins]).unsqueeze(1), h, w)

    h = x.unsqueeze(0).expand(len(mlps), *x.shape)
    for i in range(len(mlps[0].residual)):
        blocks = [m.residual[i] for m in mlps]
        y = lin(act(h, [b.activation1 for b in blocks]), [b.linear1 for b in blocks])
        h = h + lin(act(y, [b.activation2 for b in blocks]), [b.linear2 for b in blocks])
    return list(lin(act(h, [m.activation for m in mlps]), [m.linear for m in mlps]).unbind(0))


class NuclearEmbedding(nn.Module):
    """``e_Z = M d_Z + e~_Z``, both zero at start."""

    def __init__(self, n_features: int):
        super().__init__()
        self.register_buffer("electron_config", torch.tensor(electron_configurations(),
                                                              dtype=torch.get_default_dtype()), persistent=False)
        self.element_embedding = nn.Parameter(torch.zeros(MAX_Z, n_features))
        self.config_linear = nn.Linear(20, n_features, bias=False)
        nn.init.zeros_(self.config_linear.weight)

    def forward(self, z: Tensor) -> Tensor:
        return (self.element_embedding + self.config_linear(self.electron_config))[z]


class ElectronicEmbedding(nn.Module):
    """Total charge (``charge=True``: separate keys/values for + and -) or unpaired electrons spread
    over the atoms by ``softplus(q_i . k / sqrt(F))`` weights normalised per structure."""

    def __init__(self, n_features: int, n_residual: int, charge: bool):
        super().__init__()
        self.charge = charge
        n_in = 2 if charge else 1
        self.linear_q = nn.Linear(n_features, n_features)
        self.linear_k = nn.Linear(n_in, n_features, bias=False)
        self.linear_v = nn.Linear(n_in, n_features, bias=False)
        self.resmlp = ResidualMLP(n_features, n_residual, bias=False, zero_init=True)
        for lin in (self.linear_q, self.linear_k, self.linear_v):
            glorot_orthogonal_(lin.weight)
        nn.init.zeros_(self.linear_q.bias)

    def forward(self, e_z: Tensor, psi: Tensor, batch: Tensor, num_graphs: int) -> Tensor:
        e = F.relu(torch.stack([psi, -psi], -1)) if self.charge else psi.abs().unsqueeze(-1)
        k = gather_rows(self.linear_k(e / e.clamp(min=1.0)), batch)
        v = gather_rows(self.linear_v(e), batch)
        q = self.linear_q(e_z)
        a = F.softplus((k * q).sum(-1) / math.sqrt(q.shape[-1]), threshold=40.0 if q.dtype == torch.float64 else 20.0)
        norm = gather_rows(scatter_sum(a, batch, num_graphs), batch)
        return self.resmlp((a / (norm + 1e-8)).unsqueeze(-1) * v)


class LocalInteraction(nn.Module):
    """s-, p- and d-like messages ``sum_j resmlp(x_j) G rho(r_ij) Y_l(r_ij)``; the p and d sums
    enter through the invariant pair products ``<P1 p, P2 p>``, ``<D1 d, D2 d>``."""

    def __init__(self, n_features: int, n_rbf: int, n_residual: int):
        super().__init__()
        self.n_features = n_features
        self.radial_s = nn.Linear(n_rbf, n_features, bias=False)
        self.radial_p = nn.Linear(n_rbf, n_features, bias=False)
        self.radial_d = nn.Linear(n_rbf, n_features, bias=False)
        self.resmlp_c = ResidualMLP(n_features, n_residual)
        self.resmlp_s = ResidualMLP(n_features, n_residual)
        self.resmlp_p = ResidualMLP(n_features, n_residual)
        self.resmlp_d = ResidualMLP(n_features, n_residual)
        self.projection_p = nn.Linear(n_features, 2 * n_features, bias=False)
        self.projection_d = nn.Linear(n_features, 2 * n_features, bias=False)
        self.resmlp_l = ResidualMLP(n_features, n_residual, zero_init=True)
        for lin in (self.radial_s, self.radial_p, self.radial_d, self.projection_p, self.projection_d):
            glorot_orthogonal_(lin.weight)

    def forward(self, x, rho, y1, y2, src, dst, use_p: bool, use_d: bool) -> Tensor:
        n = x.shape[0]
        nets = [self.resmlp_c, self.resmlp_s] + ([self.resmlp_p] if use_p else []) + ([self.resmlp_d] if use_d else [])
        outs = residual_mlps(x, nets)
        total = outs[0] + scatter_sum(self.radial_s(rho) * gather_rows(outs[1], src), dst, n)
        if use_p:
            g = (self.radial_p(rho) * gather_rows(outs[2], src)).unsqueeze(1) * y1.unsqueeze(-1)
            a, b = torch.split(self.projection_p(scatter_sum(g, dst, n)), self.n_features, -1)
            total = total + (a * b).sum(1)
        if use_d:
            g = (self.radial_d(rho) * gather_rows(outs[-1], src)).unsqueeze(1) * y2.unsqueeze(-1)
            a, b = torch.split(self.projection_d(scatter_sum(g, dst, n)), self.n_features, -1)
            total = total + (a * b).sum(1)
        return self.resmlp_l(total)


def _pad(x: Tensor, flat: Tensor, b: int, n_max: int, fill: float) -> Tensor:
    out = x.new_full((b * n_max, x.shape[-1]), fill)
    return out.index_copy(0, flat, x).view(b, n_max, x.shape[-1])


def _unpad(y: Tensor, flat: Tensor) -> Tensor:
    return gather_rows(y.reshape(-1, y.shape[-1]), flat)


def structure_slots(batch: Tensor, num_graphs: int) -> Tuple[Tensor, int]:
    """Index of every atom within its structure and the largest structure size."""
    counts = torch.bincount(batch, minlength=num_graphs)
    starts = torch.cumsum(counts, 0) - counts
    order = torch.argsort(batch, stable=True)
    slot = torch.empty_like(batch)
    slot[order] = torch.arange(batch.shape[0], device=batch.device) - starts[batch[order]]
    return slot, int(counts.max()) if counts.numel() else 0


class NonlocalInteraction(nn.Module):
    """Self-attention over the atoms of each structure: FAVOR+ positive random features (``omega``
    drawn once) or exact softmax (``n_random_features=None``)."""

    def __init__(self, n_features: int, n_residual: int, n_random_features: Optional[int],
                 generator: Optional[torch.Generator] = None):
        super().__init__()
        self.resmlp_q = ResidualMLP(n_features, n_residual, zero_init=True)
        self.resmlp_k = ResidualMLP(n_features, n_residual, zero_init=True)
        self.resmlp_v = ResidualMLP(n_features, n_residual, zero_init=True)
        self.exact = n_random_features is None
        omega = (torch.zeros(n_features, 0, dtype=torch.float64) if self.exact
                 else orthogonal_random_features(int(n_random_features), n_features, generator))
        self.register_buffer("omega", omega.to(torch.get_default_dtype()))

    def _phi(self, x: Tensor, u: Tensor, shift: Tensor) -> Tensor:
        h = (x * x).sum(-1, keepdim=True) / (2.0 * math.sqrt(x.shape[-1]))
        return (torch.exp(u - h - shift) + 1e-4) / math.sqrt(self.omega.shape[-1])

    def forward(self, x: Tensor, batch: Tensor, num_graphs: int, slot: Tensor, n_max: int) -> Tensor:
        q, k, v = residual_mlps(x, [self.resmlp_q, self.resmlp_k, self.resmlp_v])
        flat = batch * n_max + slot
        if self.exact:
            return self._exact(q, k, v, flat, num_graphs, n_max)
        scale = x.shape[-1] ** 0.25
        u_q, u_k = (q / scale) @ self.omega, (k / scale) @ self.omega
        phi_q = self._phi(q, u_q, u_q.max(-1, keepdim=True).values)
        if num_graphs == 1:
            phi_k = self._phi(k, u_k, u_k.max())
            return (phi_q @ (phi_k.t() @ v)) / (phi_q @ phi_k.sum(0) + 1e-8).unsqueeze(-1)
        shift = gather_rows(_pad(u_k, flat, num_graphs, n_max, -math.inf).flatten(1).max(1).values, batch)
        phi_k = self._phi(k, u_k, shift.unsqueeze(-1))
        pq, pk = _pad(phi_q, flat, num_graphs, n_max, 0.0), _pad(phi_k, flat, num_graphs, n_max, 0.0)
        num = _unpad(torch.bmm(pq, torch.bmm(pk.transpose(1, 2), _pad(v, flat, num_graphs, n_max, 0.0))), flat)
        den = _unpad((pq * pk.sum(1, keepdim=True)).sum(-1, keepdim=True), flat).squeeze(-1)
        return num / (den + 1e-8).unsqueeze(-1)

    def _exact(self, q, k, v, flat, b: int, n_max: int) -> Tensor:
        pq, pk, pv = (_pad(t, flat, b, n_max, 0.0) for t in (q, k, v))
        valid = torch.zeros(b * n_max, dtype=torch.bool, device=q.device).index_fill(0, flat, True).view(b, n_max)
        dot = torch.bmm(pq, pk.transpose(1, 2))
        mask = valid.unsqueeze(1) & valid.unsqueeze(2)
        shift = torch.where(mask, dot, -math.inf).flatten(1).max(1).values
        a = torch.where(mask, torch.exp((dot - shift[:, None, None]) / math.sqrt(q.shape[-1])), 0.0)
        return _unpad(torch.bmm(a / (a.sum(-1, keepdim=True) + 1e-8), pv), flat)


class InteractionModule(nn.Module):
    """``x~ = residual(x)``, ``x' = residual(x~ + l + n)``, ``y = resmlp(x')``."""

    def __init__(self, n_features: int, n_rbf: int, n_residual: int, nonlocal_: bool,
                 n_random_features: Optional[int], generator: Optional[torch.Generator]):
        super().__init__()
        self.residual_pre = nn.ModuleList(ResidualBlock(n_features) for _ in range(n_residual))
        self.local_interaction = LocalInteraction(n_features, n_rbf, n_residual)
        self.nonlocal_interaction = (NonlocalInteraction(n_features, n_residual, n_random_features, generator)
                                     if nonlocal_ else None)
        self.residual_post = nn.ModuleList(ResidualBlock(n_features) for _ in range(n_residual))
        self.resmlp_y = ResidualMLP(n_features, n_residual)

    def forward(self, x, rho, y1, y2, src, dst, batch, num_graphs, slot, n_max, use_p, use_d, use_nonlocal):
        for block in self.residual_pre:
            x = block(x)
        h = x + self.local_interaction(x, rho, y1, y2, src, dst, use_p, use_d)
        if self.nonlocal_interaction is not None and use_nonlocal:
            h = h + self.nonlocal_interaction(x, batch, num_graphs, slot, n_max)
        for block in self.residual_post:
            h = block(h)
        return h, self.resmlp_y(h)


class ZBLRepulsion(nn.Module):
    """``k_e sum_{i<j} Z_i Z_j / r f_c(r) sum_k c_k exp(-a_k r (Z_i^p + Z_j^p) / d)`` with softplus-
    positive parameters starting at the universal ZBL screening; ``c`` normalised to sum 1."""

    def __init__(self):
        super().__init__()
        self.k_e = COULOMB_CONSTANT
        dt = torch.get_default_dtype()
        self._adiv = nn.Parameter(torch.tensor(float(softplus_inverse(1.0 / (0.8854 * BOHR))), dtype=dt))
        self._apow = nn.Parameter(torch.tensor(float(softplus_inverse(0.23)), dtype=dt))
        self._c = nn.Parameter(torch.tensor(softplus_inverse(np.array([0.18180, 0.50990, 0.28020, 0.02817])), dtype=dt))
        self._a = nn.Parameter(torch.tensor(softplus_inverse(np.array([3.20000, 0.94230, 0.40280, 0.20160])), dtype=dt))

    def forward(self, zf: Tensor, r: Tensor, fcut: Tensor, src: Tensor, dst: Tensor) -> Tensor:
        zp = zf ** F.softplus(self._apow)
        a = (zp[dst] + zp[src]) * F.softplus(self._adiv)
        c = F.softplus(self._c)
        screen = (c / c.sum() * torch.exp(-F.softplus(self._a) * (a * r).unsqueeze(-1))).sum(-1)
        return scatter_sum(0.5 * self.k_e * zf[dst] * zf[src] / r * screen * fcut, dst, zf.shape[0])


class DampedCoulomb(nn.Module):
    """``k_e q_i q_j [f / sqrt(r^2 + 1) + (1 - f) / r]`` with ``f`` switching off between
    ``r_c / 4`` and ``3 r_c / 4``; with ``lr_cutoff`` both kernels are shifted to zero value and
    slope there."""

    def __init__(self, cutoff: float, lr_cutoff: Optional[float]):
        super().__init__()
        self.k_e = COULOMB_CONSTANT
        self.r_on, self.r_off = 0.25 * float(cutoff), 0.75 * float(cutoff)
        self.lr_cutoff = None if lr_cutoff is None else float(lr_cutoff)

    def kernel(self, r: Tensor) -> Tensor:
        f = smooth_switch(r, self.r_on, self.r_off)
        bare, soft = 1.0 / r, 1.0 / torch.sqrt(r * r + 1.0)
        lr = self.lr_cutoff
        if lr is not None:
            c3 = (lr * lr + 1.0) ** 1.5
            inside = r < lr
            bare = torch.where(inside, bare + r / (lr * lr) - 2.0 / lr, 0.0)
            soft = torch.where(inside, soft + r * lr / c3 - (2.0 * lr * lr + 1.0) / c3, 0.0)
        return f * soft + (1.0 - f) * bare

    def forward(self, q: Tensor, src: Tensor, dst: Tensor, r: Tensor) -> Tensor:
        return scatter_sum(0.5 * self.k_e * q[src] * q[dst] * self.kernel(r), dst, q.shape[0])

    def damping(self, q: Tensor, src: Tensor, dst: Tensor, r: Tensor) -> Tensor:
        """The short-range correction ``k_e q_i q_j f (1 / sqrt(r^2 + 1) - 1 / r)`` (Ewald path)."""
        f = smooth_switch(r, self.r_on, self.r_off)
        pair = 0.5 * self.k_e * q[src] * q[dst] * f * (1.0 / torch.sqrt(r * r + 1.0) - 1.0 / r)
        return scatter_sum(pair, dst, q.shape[0])


class ChargeD4(nn.Module):
    """Two-body D4 with the model's charges: C6 from the charge- and CN-dependent polarizabilities
    (Casimir-Polder), ``C8 = 3 C6 Q_i Q_j``, BJ damping; learnable ``s8, a1, a2`` and the reference-
    charge scale ``s_q`` (softplus-positive, Hartree-Fock starting values); ``s6 = 1`` fixed."""

    def __init__(self, s6: float = 1.0, s8: float = 1.61679827, a1: float = 0.44959224, a2: float = 3.35743605,
                 lr_cutoff: Optional[float] = None, ga: float = 3.0, gc: float = 2.0, wf: float = 6.0):
        super().__init__()
        self.lr_cutoff = None if lr_cutoff is None else float(lr_cutoff)
        self.ga, self.gc, self.wf = float(ga), float(gc), float(wf)
        ref = load_tables("d4_reference.npz")
        dt = torch.get_default_dtype()
        zz = np.arange(ref["r4r2_raw"].shape[0], dtype=np.float64)
        tables = {
            "rcov": 4.0 / 3.0 * ref["covalent_radius_aa"] / BOHR, "en": ref["pauling_en"], "zeff": ref["zeff"],
            "hardness": ref["hardness"], "r4r2": np.sqrt(0.5 * ref["r4r2_raw"] * np.sqrt(zz)),
            "refcn": ref["refcn"], "refq": ref["refq"], "cp_weights": np.array(CP_WEIGHTS),
            "refh": ref["refh"], "sscale": ref["sscale"], "secaiw": ref["secaiw"], "ascale": ref["ascale"],
            "alphaiw": ref["alphaiw"], "hcount": ref["hcount"]}
        for name, a in tables.items():
            self.register_buffer(name, torch.tensor(np.asarray(a, dtype=np.float64), dtype=dt), persistent=False)
        for name in ("nref", "ngw", "refsys"):
            self.register_buffer(name, torch.tensor(ref[name], dtype=torch.long), persistent=False)
        self.n_gauss = int(np.max(ref["ngw"]))
        self.register_buffer("_s6", torch.tensor(float(softplus_inverse(s6)), dtype=dt))
        self._s8 = nn.Parameter(torch.tensor(float(softplus_inverse(s8)), dtype=dt))
        self._a1 = nn.Parameter(torch.tensor(float(softplus_inverse(a1)), dtype=dt))
        self._a2 = nn.Parameter(torch.tensor(float(softplus_inverse(a2)), dtype=dt))
        self._scaleq = nn.Parameter(torch.tensor(float(softplus_inverse(1.0)), dtype=dt))

    def _zeta(self, hardness: Tensor, qref: Tensor, qmod: Tensor) -> Tensor:
        pos = qmod > 1e-8
        safe = torch.where(pos, qmod, 1.0)
        return torch.where(pos, torch.exp(self.ga * (1.0 - torch.exp(hardness * self.gc * (1.0 - qref / safe)))),
                           math.exp(self.ga))

    def reference_polarizabilities(self, scale_q: Tensor) -> Tensor:
        """``(23, 7, Z)`` reference ``alpha(i w)`` with the secondary systems' hydrogen charges scaled."""
        present = self.refsys > 0
        sec = torch.where(present, self.refsys, 0)
        zx = self.zeff[sec]
        scale = self._zeta(self.hardness[sec], zx, self.refh * scale_q + zx)
        alpha = self.ascale * (self.alphaiw - self.hcount * self.sscale[sec] * self.secaiw[:, sec] * scale)
        return torch.where(present, alpha.clamp(min=0.0), 0.0)

    def forward(self, z: Tensor, q: Tensor, src: Tensor, dst: Tensor, r_ang: Tensor) -> Tensor:
        n = z.shape[0]
        r = r_ang / BOHR
        zi, zj = z[dst], z[src]
        rc = self.rcov[zi] + self.rcov[zj]
        count = 0.5 * (1.0 + torch.erf(-KCN * (r - rc) / rc)) * K4 * torch.exp(
            -((self.en[zi] - self.en[zj]).abs() + K5) ** 2 / K6)
        lr = self.lr_cutoff
        if lr is not None:
            count = count * smooth_switch(r, lr / BOHR - BOHR, lr / BOHR)
        cn = scatter_sum(count, dst, n)
        refcn = self.refcn[:, z].t()
        valid = torch.arange(refcn.shape[1], device=z.device)[None, :] < self.nref[z][:, None]
        w = gaussian_reference_weights(cn, refcn, valid, self.wf, self.ngw[:, z].t(), 1e-8, n_gauss=self.n_gauss)
        scale_q = F.softplus(self._scaleq)
        zeff = self.zeff[z][:, None]
        zeta = self._zeta(self.hardness[z][:, None], zeff + self.refq[:, z].t() * scale_q, zeff + q[:, None])
        alpha_iw = torch.einsum("nr,krn->nk", w * zeta, self.reference_polarizabilities(scale_q)[:, :, z])
        c6 = (3.0 / math.pi) * (alpha_iw[dst] * alpha_iw[src] * self.cp_weights).sum(-1)
        rr = 3.0 * self.r4r2[zi] * self.r4r2[zj]
        r0 = F.softplus(self._a1) * torch.sqrt(rr) + F.softplus(self._a2)
        r0_6, r0_8 = r0 ** 6, r0 ** 8
        t6, t8 = 1.0 / (r ** 6 + r0_6), 1.0 / (r ** 8 + r0_8)
        if lr is not None:
            cut = lr / BOHR
            c6c, c8c = cut ** 6, cut ** 8
            tail = r / cut - 1.0
            inside = r < cut
            t6 = torch.where(inside, t6 - 1.0 / (c6c + r0_6) + 6.0 * c6c / (c6c + r0_6) ** 2 * tail, 0.0)
            t8 = torch.where(inside, t8 - 1.0 / (c8c + r0_8) + 8.0 * c8c / (c8c + r0_8) ** 2 * tail, 0.0)
        pair = -0.5 * HARTREE * c6 * (F.softplus(self._s6) * t6 + F.softplus(self._s8) * rr * t8)
        return scatter_sum(pair, dst, n)


@register_model("spookynet")
class SpookyNet(InteratomicPotential):
    """SpookyNet: ``E_i = E_nn + E_rep + E_ele + E_vdw`` with charges summing to the total charge.

    Defaults are the paper's (F = 128, T = 6, K = 16, cutoff 10 bohr, FAVOR+ with F features, all
    three physical terms). Inputs beyond positions and species: ``total_charge`` (neutral when
    absent) and ``spin_multiplicity`` (singlet when absent). ``lr_cutoff`` truncates the
    electrostatics and dispersion (needed for periodic structures; otherwise they run over all
    pairs of each structure); ``ewald=True`` Ewald-sums the periodic structures' Coulomb part.
    """

    head_modules = ("output", "atom_ref", "charge_ref")

    def __init__(self, n_features: int = 128, n_interactions: int = 6, n_rbf: int = 16, cutoff: float = 10.0 * BOHR,
                 lr_cutoff: Optional[float] = None, n_residual: int = 1, charge_embedding: bool = True,
                 spin_embedding: bool = True, nonlocal_interactions: bool = True, attention: str = "favor",
                 n_random_features: Optional[int] = None, zbl_repulsion: bool = True, electrostatics: bool = True,
                 d4_dispersion: bool = True, exp_weighting: bool = False, ewald: bool = False,
                 ewald_accuracy: float = 1.0e-6, seed: Optional[int] = None, species=None, atomic_energies=None):
        super().__init__()
        if attention not in ("favor", "exact"):
            raise ValueError(f"attention must be 'favor' or 'exact', got {attention!r}")
        if ewald and lr_cutoff is None:
            raise ValueError("ewald=True needs lr_cutoff (the real-space cutoff)")
        self.local_cutoff = float(cutoff)
        self.lr_cutoff = None if lr_cutoff is None else float(lr_cutoff)
        self.cutoff = max(self.local_cutoff, self.lr_cutoff or 0.0)
        self.species = [int(s) for s in species] if species is not None else None
        self.n_features = self.node_feature_dim = n_features
        self.use_p_orbitals = self.use_d_orbitals = self.use_nonlocal = True
        self.ewald = bool(ewald)
        self.ewald_alpha, self.ewald_k_cutoff = (ewald_parameters(self.lr_cutoff, float(ewald_accuracy))
                                                 if self.ewald else (0.0, 0.0))
        gen = torch.Generator().manual_seed(int(seed)) if seed is not None else None
        m = None if attention == "exact" else int(n_random_features or n_features)
        self.nuclear_embedding = NuclearEmbedding(n_features)
        self.charge_embedding = ElectronicEmbedding(n_features, n_residual, True) if charge_embedding else None
        self.spin_embedding = ElectronicEmbedding(n_features, n_residual, False) if spin_embedding else None
        self.radial_basis = ExponentialBernsteinRBF(n_rbf, exp_weighting=exp_weighting)
        self.interactions = nn.ModuleList(
            InteractionModule(n_features, n_rbf, n_residual, nonlocal_interactions, m, gen)
            for _ in range(n_interactions))
        self.output = nn.Linear(n_features, 2, bias=False)
        glorot_orthogonal_(self.output.weight)
        self.atom_ref = nn.Embedding(MAX_Z, 1)
        self.charge_ref = nn.Embedding(MAX_Z, 1)
        nn.init.zeros_(self.atom_ref.weight)
        nn.init.zeros_(self.charge_ref.weight)
        self.repulsion = ZBLRepulsion() if zbl_repulsion else None
        self.electrostatics = DampedCoulomb(self.local_cutoff, self.lr_cutoff) if electrostatics else None
        self.dispersion = ChargeD4(lr_cutoff=self.lr_cutoff) if d4_dispersion else None
        if atomic_energies is not None:
            if species is None:
                raise ValueError("species is required to map atomic_energies")
            self.set_atomic_energies(species, atomic_energies)

    def receptive_field(self):
        return None

    def set_atomic_energies(self, species, values) -> None:
        ae = torch.as_tensor(values, dtype=self.atom_ref.weight.dtype)
        species = [int(s) for s in species]
        if ae.numel() != len(species):
            raise ValueError(f"got {ae.numel()} atomic energies for {len(species)} species")
        with torch.no_grad():
            self.atom_ref.weight[torch.tensor(species), 0] = ae

    def _cutoff_fn(self, r: Tensor) -> Tensor:
        x = (r / self.local_cutoff).clamp(0.0, 1.0 - 1e-6)
        return torch.exp(1.0 - 1.0 / (1.0 - x * x))

    def _long_range_pairs(self, edge_index, r_all, pos, batch, periodic: bool):
        if self.lr_cutoff is not None:
            keep = (r_all < self.lr_cutoff).nonzero().squeeze(1)
            return edge_index[0][keep], edge_index[1][keep], r_all[keep]
        if periodic:
            raise ValueError("SpookyNet sums the long-range terms over all pairs of a molecule; "
                             "periodic structures need lr_cutoff")
        dst, src = all_pairs(batch)
        return src, dst, torch.linalg.norm(pos[dst] - pos[src], dim=-1)

    def _evaluate(self, z, edge_index, edge_vec, pos, cell, pbc, batch, num_graphs, total_charge, n_unpaired):
        dtype = self.output.weight.dtype
        n = z.shape[0]
        r_all = torch.linalg.norm(edge_vec, dim=-1)
        local = (r_all < self.local_cutoff).nonzero().squeeze(1)
        src, dst, r = edge_index[0][local], edge_index[1][local], r_all[local]
        u = -edge_vec[local] / r.unsqueeze(-1)          # r_ij = r_j - r_i, the negative of the edge vector
        ux, uy, uz = u.unbind(-1)
        s3 = math.sqrt(3.0)
        y1 = torch.stack([uy, uz, ux], -1)
        y2 = torch.stack([s3 * ux * uy, s3 * uy * uz, 0.5 * (3.0 * uz * uz - 1.0), s3 * ux * uz,
                          0.5 * s3 * (ux * ux - uy * uy)], -1)
        fcut = self._cutoff_fn(r)
        rho = self.radial_basis(r) * fcut.unsqueeze(-1)
        e_z = self.nuclear_embedding(z)
        x = e_z
        if self.charge_embedding is not None:
            x = x + self.charge_embedding(e_z, total_charge, batch, num_graphs)
        if self.spin_embedding is not None:
            x = x + self.spin_embedding(e_z, n_unpaired, batch, num_graphs)
        if num_graphs > 1:
            slot, n_max = structure_slots(batch, num_graphs)
        else:
            slot, n_max = torch.arange(n, device=z.device), n
        f = torch.zeros_like(x)
        for module in self.interactions:
            x, y = module(x, rho, y1, y2, src, dst, batch, num_graphs, slot, n_max,
                          self.use_p_orbitals, self.use_d_orbitals, self.use_nonlocal)
            f = f + y
        out = self.output(f)
        e_nn = out[:, 0] + self.atom_ref(z).squeeze(-1)
        q = out[:, 1] + self.charge_ref(z).squeeze(-1)
        counts = scatter_sum(torch.ones_like(e_nn), batch, num_graphs)
        q = q + gather_rows((total_charge - scatter_sum(q, batch, num_graphs)) / counts, batch)
        zero = torch.zeros_like(e_nn)
        e_rep = self.repulsion(z.to(dtype), r, fcut, src, dst) if self.repulsion is not None else zero
        e_ele, e_vdw = zero, zero
        if self.electrostatics is not None or self.dispersion is not None:
            periodic_atoms = torch.zeros(n, dtype=torch.bool, device=z.device)
            if cell is not None and pbc is not None:
                periodic_atoms = pbc.any(1)[batch]
            any_periodic = bool(periodic_atoms.any())
            ls, ld, lr_r = self._long_range_pairs(edge_index, r_all, pos, batch, any_periodic)
            if self.electrostatics is not None:
                if self.ewald and any_periodic:
                    e_ele = self._ewald(q, pos, cell, pbc, batch, num_graphs, ls, ld, lr_r, periodic_atoms)
                else:
                    e_ele = self.electrostatics(q, ls, ld, lr_r)
            if self.dispersion is not None:
                e_vdw = self.dispersion(z, q, ls, ld, lr_r)
        return {"node_features": f, "node_energy": e_nn + e_rep + e_ele + e_vdw, "charges": q,
                "node_repulsion": e_rep, "node_electrostatics": e_ele, "node_dispersion": e_vdw}

    def _ewald(self, q, pos, cell, pbc, batch, num_graphs, src, dst, r, periodic_atoms):
        elec = self.electrostatics
        on = periodic_atoms[dst]
        node = elec(q, src[~on], dst[~on], r[~on]) + elec.damping(q, src[on], dst[on], r[on])
        for i in range(num_graphs):
            flags = pbc[i]
            if not bool(flags.any()):
                continue
            if not bool(flags.all()):
                raise ValueError("ewald=True needs structures periodic in all three directions")
            mask = batch == i
            idx = mask.nonzero().squeeze(1)
            sel = mask[dst]
            remap = torch.cumsum(mask.long(), 0) - 1
            part = coulomb_ewald(q[idx], pos[idx], cell[i], torch.stack([remap[src[sel]], remap[dst[sel]]]),
                                 r[sel], self.ewald_alpha, self.lr_cutoff, self.ewald_k_cutoff, elec.k_e)
            node = node.index_add(0, idx, part.to(node.dtype))
        return node

    def forward(self, data: AtomicGraph) -> dict:
        dtype = self.output.weight.dtype
        b = data.num_graphs
        dev = data.atomic_numbers.device
        q_tot = data.total_charge.to(dtype) if data.total_charge is not None else torch.zeros(b, dtype=dtype, device=dev)
        unpaired = (data.spin_multiplicity.to(dtype) - 1.0 if data.spin_multiplicity is not None
                    else torch.zeros(b, dtype=dtype, device=dev))
        out = self._evaluate(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.pos.to(dtype),
                             data.cell, data.pbc, data.batch, b, q_tot, unpaired)
        q = out["charges"]
        terms = scatter_sum(torch.stack([out["node_repulsion"], out["node_electrostatics"], out["node_dispersion"]],
                                        -1).to(torch.float64), data.batch, b)
        return {"node_energy": out["node_energy"], "energy": self.aggregate_energy(out["node_energy"], data),
                "node_features": out["node_features"], "charges": q,
                "dipole": scatter_sum(q.unsqueeze(-1) * data.pos.to(dtype), data.batch, b),
                "energy_repulsion": terms[:, 0], "energy_electrostatics": terms[:, 1],
                "energy_dispersion": terms[:, 2]}

    @classmethod
    def from_config(cls, cfg) -> "SpookyNet":
        e = dict(cfg.extra or {})
        keys = ("lr_cutoff", "n_residual", "charge_embedding", "spin_embedding", "nonlocal_interactions", "attention",
                "n_random_features", "zbl_repulsion", "electrostatics", "d4_dispersion", "exp_weighting", "ewald",
                "ewald_accuracy", "seed", "species", "atomic_energies")
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf, cutoff=cfg.cutoff,
                   **{k: e[k] for k in keys if k in e})

    @classmethod
    def from_reference_checkpoint(cls, source) -> "SpookyNet":
        """A model from a file written by the SpookyNet authors' code (``SpookyNet.save``): the
        hyperparameters, renamed parameters and the radial weights in the paper's order."""
        state = source if isinstance(source, dict) else torch.load(source, map_location="cpu", weights_only=True)
        hp = {k: v for k, v in state.items() if k != "state_dict"}
        for key, want, legacy in (("activation", "swish", "swish"), ("basis_functions", "exp-bernstein", "exp-bernstein"),
                                  ("use_irreps", True, False), ("use_nonlinear_embedding", False, True),
                                  ("Zmax", MAX_Z, MAX_Z)):
            if hp.get(key, legacy) != want:
                raise ValueError(f"reference checkpoint has {key}={hp.get(key)!r}; only {key}={want!r} is supported")
        depths = {int(v) for k, v in hp.items() if k.startswith("num_residual")}
        if len(depths) > 1:
            raise ValueError(f"different residual depths {sorted(depths)} are not supported")
        sd = state["state_dict"]
        prev = torch.get_default_dtype()
        torch.set_default_dtype(sd["output.weight"].dtype)
        try:
            model = cls(n_features=int(hp["num_features"]), n_interactions=int(hp["num_modules"]),
                        n_rbf=int(hp["num_basis_functions"]), cutoff=float(hp["cutoff"]), lr_cutoff=hp.get("lr_cutoff"),
                        n_residual=depths.pop() if depths else 1, zbl_repulsion=bool(hp["use_zbl_repulsion"]),
                        electrostatics=bool(hp["use_electrostatics"]), d4_dispersion=bool(hp["use_d4_dispersion"]),
                        exp_weighting=bool(hp["exp_weighting"]))
        finally:
            torch.set_default_dtype(prev)
        model.load_state_dict(reference_state_dict(sd))
        return model.eval()


# authors' parameter names -> these (applied in order)
_RENAMES = (
    (r"\.stack\.", "."), (r"^magmom_embedding\.", "spin_embedding."), (r"^module\.", "interactions."),
    (r"_embedding\.resblock\.", "_embedding.resmlp."),
    (r"\.local_interaction\.resblock_x\.", ".local_interaction.resmlp_c."),
    (r"\.resblock_([spdqkv])\.", r".resmlp_\1."), (r"\.local_interaction\.resblock\.", ".local_interaction.resmlp_l."),
    (r"^(interactions\.\d+)\.resblock\.", r"\1.resmlp_y."), (r"\.attention\.omega$", ".omega"),
    (r"^zbl_repulsion_energy\.", "repulsion."), (r"^d4_dispersion_energy\.", "dispersion."),
    (r"^radial_basis_functions\._alpha$", "radial_basis.gamma_raw"),
)
_SCALARS = ("repulsion._adiv", "repulsion._apow", "dispersion._s6", "dispersion._s8", "dispersion._a1",
            "dispersion._a2", "dispersion._scaleq", "radial_basis.gamma_raw")
_DROPPED = re.compile(r"keep_prob|nuclear_embedding\.(electron_config|embedding)|radial_basis_functions\.(logc|n|v)"
                      r"|d4_dispersion_energy\.(?!_s6$|_s8$|_a1$|_a2$|_scaleq$).*")


def reference_state_dict(sd: Dict[str, Tensor]) -> Dict[str, Tensor]:
    """The authors' state dict under this model's names (tables dropped, element biases split, the
    four ZBL coefficients stacked, radial weights reversed to the paper's order)."""
    out: Dict[str, Tensor] = {}
    zbl: Dict[str, List[Tensor]] = {"c": [], "a": []}
    for key in sorted(sd):
        v = sd[key]
        if key == "element_bias":
            out["atom_ref.weight"], out["charge_ref.weight"] = v[:, :1].clone(), v[:, 1:].clone()
            continue
        if _DROPPED.fullmatch(key):
            continue
        coef = re.fullmatch(r"zbl_repulsion_energy\._([ca])\d", key)
        if coef is not None:
            zbl[coef.group(1)].append(v.reshape(1))
            continue
        new = key
        for pat, rep in _RENAMES:
            new = re.sub(pat, rep, new)
        if re.search(r"\.radial_[spd]\.weight$", new):
            v = v.flip(-1)
        out[new] = v.reshape(()) if new in _SCALARS else v
    if zbl["c"]:
        out["repulsion._c"], out["repulsion._a"] = torch.cat(zbl["c"]), torch.cat(zbl["a"])
    return out
