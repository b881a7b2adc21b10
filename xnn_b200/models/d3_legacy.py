"""The D3(BJ) pair dispersion of the PhysNet / BAMBOO codes (two-body only, Grimme's original
2010 reference systems, optional force-shifted cutoff with a one-bohr C2 taper on the counts).

Per directed edge ``(i <- j)``: ``CN_i = sum_j 1 / (1 + exp(-16 (R_ij / r - 1))) taper(r)``;
``C6_ij`` the Gaussian-weighted (``exp(-4 dCN^2)``) average of the reference ``C6``;
``C8 = 3 C6 Q_i Q_j``; ``E_i = -1/2 sum_j (s6 C6 f6 + s8 C8 f8)`` with ``f_n = 1 / (r^n + R0^n)``,
``R0 = a1 sqrt(C8 / C6) + a2`` (atomic units). Behaviour follows the reference
(``src/xnn/common/models/d3.py:208-471``); the reference systems come from its data file, and the
radii and ``sqrt(Q)`` factors are computed from that file in float64 (the PhysNet TF code keeps
float32 roundings of them, a relative difference below 1e-6).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch
from torch import Tensor

from .dispersion import load_tables

AUTOANG = 0.52917726
AUTOEV = 27.21138505
S6, S8, A1, A2 = 1.0, 0.9171, 0.3385, 2.8830
_K1, _K3 = 16.0, -4.0


def reference_sets(references: str = "2010") -> dict:
    """``nref``, ``refcn (7, Z)`` and ``c6 (7, 7, Z, Z)`` of one reference set (``"2010"``:
    Grimme's original systems, nothing beyond the original last element; ``"2024"``: current)."""
    t = load_tables("d3_reference.npz")
    nref, refcn, c6 = t["nref"].copy(), t["refcn"].copy(), t["c6"].copy()
    if references == "2010":
        zs = t["original_z"]
        nref[zs] = t["original_nref"]
        refcn[:, zs] = t["original_refcn"]
        c6[:, :, zs, :] = t["original_c6"]
        c6[:, :, :, zs] = t["original_c6"].transpose(1, 0, 3, 2)
        beyond = int(t["original_max_z"]) + 1
        nref[beyond:] = 0
        refcn[:, beyond:] = -1.0
        c6[:, :, beyond:, :] = 0.0
        c6[:, :, :, beyond:] = 0.0
    elif references != "2024":
        raise ValueError(f"references must be '2010' or '2024', got {references!r}")
    return {"nref": nref, "refcn": refcn, "c6": c6, "covalent_radius_aa": t["covalent_radius_aa"],
            "r4r2_raw": t["r4r2_raw"]}


def legacy_tables(references: str = "2010", max_z: int = 95):
    """``(c6ab (Z, Z, R, R, 3), rcov (Z,), r2r4 (Z,))``: per element pair and reference pair the
    ``(C6, CN_i, CN_j)`` (``-1`` in unused slots, zero for ``Z = 0``), the 4/3-scaled covalent radii
    in bohr and the ``sqrt(Q)`` factors."""
    tab = reference_sets(references)
    nref = tab["nref"][:max_z]
    n_slots = int(nref.max())
    valid = np.arange(n_slots)[None, :] < nref[:, None]
    mask = valid[:, None, :, None] & valid[None, :, None, :]
    c6 = tab["c6"][:n_slots, :n_slots, :max_z, :max_z].transpose(2, 3, 0, 1)
    cn = tab["refcn"][:n_slots, :max_z].T
    table = np.stack([np.where(mask, c6, -1.0),
                      np.where(mask, np.broadcast_to(cn[:, None, :, None], mask.shape), -1.0),
                      np.where(mask, np.broadcast_to(cn[None, :, None, :], mask.shape), -1.0)], -1)
    table[0] = 0.0
    table[:, 0] = 0.0
    rcov = 4.0 / 3.0 * tab["covalent_radius_aa"][:max_z] / AUTOANG
    rcov[0] = 0.0
    z = np.arange(max_z, dtype=np.float64)
    r2r4 = np.sqrt(0.5 * tab["r4r2_raw"][:max_z] * np.sqrt(z))
    return torch.from_numpy(np.ascontiguousarray(table)), torch.from_numpy(rcov), torch.from_numpy(r2r4)


def _taper(r: Tensor, cutoff: float) -> Tensor:
    u = cutoff - r
    ramp = u ** 3 * (10.0 + u * (6.0 * u - 15.0))
    return torch.where(u >= 1.0, torch.ones_like(u), torch.where(u <= 0.0, torch.zeros_like(u), ramp))


def coordination(zi: Tensor, zj: Tensor, r: Tensor, i: Tensor, n: int, cutoff: Optional[float], rcov: Tensor) -> Tensor:
    """``CN_i = sum_j 1 / (1 + exp(-16 (R_ij / r - 1)))`` (tapered over the last bohr with a cutoff)."""
    count = 1.0 / (1.0 + torch.exp(-_K1 * ((rcov[zi] + rcov[zj]).to(r.dtype) / r - 1.0)))
    if cutoff is not None:
        count = count * _taper(r, cutoff)
    return r.new_zeros(n).index_add(0, i, count)


def pair_c6(zi: Tensor, zj: Tensor, cni: Tensor, cnj: Tensor, c6ab: Tensor) -> Tensor:
    """Gaussian-weighted (``exp(-4 dCN^2)``) average of the reference ``C6`` of each pair."""
    refs = c6ab[zi, zj].to(cni.dtype)
    c6r = refs[..., 0]
    d2 = (refs[..., 1] - cni[:, None, None]) ** 2 + (refs[..., 2] - cnj[:, None, None]) ** 2
    w = torch.where(c6r > 0.0, torch.exp(_K3 * d2), torch.zeros_like(d2))
    norm = w.sum((-2, -1))
    return torch.where(norm > 0.0, (w * c6r).sum((-2, -1)) / norm,
                       torch.full_like(norm, -1.0e99 if norm.dtype == torch.float64 else float("-inf")))


def pair_dispersion(Z: Tensor, r: Tensor, i: Tensor, j: Tensor, cutoff: Optional[float], s6, s8, a1, a2,
                    c6ab: Tensor, rcov: Tensor, r2r4: Tensor) -> Tensor:
    """Per-atom D3(BJ) energies (hartree) for distances ``r`` in bohr on directed edges ``i <- j``."""
    n = Z.shape[0]
    zi, zj = Z[i], Z[j]
    cn = coordination(zi, zj, r, i, n, cutoff, rcov)
    c6 = pair_c6(zi, zj, cn[i], cn[j], c6ab)
    c8 = 3 * c6 * r2r4[zi].to(c6.dtype) * r2r4[zj].to(c6.dtype)
    r0 = a1 * torch.sqrt(c8 / c6) + a2
    r0_6 = r0 ** 6
    r0_8 = r0 ** 8
    r_6, r_8 = r ** 6, r ** 8
    if cutoff is None:
        f6, f8 = 1 / (r_6 + r0_6), 1 / (r_8 + r0_8)
    else:
        c_6, c_8 = cutoff ** 6, cutoff ** 8
        d6, d8 = c_6 + r0_6, c_8 + r0_8
        f6 = 1 / (r_6 + r0_6) - 1 / d6 + 6 * c_6 / d6 ** 2 * (r / cutoff - 1)
        f8 = 1 / (r_8 + r0_8) - 1 / d8 + 8 * c_8 / d8 ** 2 * (r / cutoff - 1)
        f6 = torch.where(r < cutoff, f6, torch.zeros_like(f6))
        f8 = torch.where(r < cutoff, f8, torch.zeros_like(f8))
    return r.new_zeros(n).index_add(0, i, -0.5 * s6 * c6 * f6 - 0.5 * s8 * c8 * f8)
