"""Point-charge electrostatics for charge-predicting models (per-atom energy shares, eV).

* ``coulomb_direct``: every pair of a structure, optionally damped by
  ``sigmoid(s (r - r_0))``;
* ``coulomb_dsf``: damped shifted force (Fennell & Gezelter 2006) within a cutoff;
* ``coulomb_ewald``: Ewald sum (real space ``erfc(a r)/r`` over the graph's edges, reciprocal
  ``4 pi / V sum_k exp(-k^2 / 4 a^2) / k^2 |S(k)|^2`` over the full ``k`` sphere, self and
  neutralising-background terms);
* ``coulomb_pme``: the same with the reciprocal part on a smooth-PME mesh (the B-spline
  spreading of :mod:`xnn_b200.ffnn.multipoles`).

The per-atom shares are ``q_i phi_i / 2``. Behaviour and parameter choices follow the reference
(``src/xnn/common/models/electrostatics.py:56-460``, ``pme.py:38``): ``a = sqrt(-ln acc) / r_c``,
``k_c = 2 a sqrt(-ln acc)``, power-of-two meshes ``2 a L / (3 acc^(1/5))``.
"""
from __future__ import annotations

import math
from typing import List, Tuple

import torch
from torch import Tensor

from ..ops.scatter import scatter_sum
from .dispersion import BOHR, HARTREE

COULOMB_CONSTANT = HARTREE * BOHR
RECIPROCAL_BUDGET = 10 ** 8


def all_pairs(batch: Tensor) -> Tuple[Tensor, Tensor]:
    same = (batch[None, :] == batch[:, None]) & ~torch.eye(batch.shape[0], dtype=torch.bool, device=batch.device)
    p = same.nonzero()
    return p[:, 0], p[:, 1]


def coulomb_direct(charges: Tensor, pos: Tensor, batch: Tensor, k_e: float = COULOMB_CONSTANT,
                   damping_midpoint: float = 0.0, damping_steepness: float = 0.0) -> Tensor:
    row, col = all_pairs(batch)
    r = torch.linalg.norm((pos.index_select(0, row) - pos.index_select(0, col)).to(charges.dtype), dim=-1)
    pair = 0.5 * k_e * charges.index_select(0, row) * charges.index_select(0, col) / r
    if damping_steepness > 0.0:
        pair = pair * torch.sigmoid(damping_steepness * (r - damping_midpoint))
    return scatter_sum(pair.to(torch.float64), row, charges.shape[0])


def coulomb_dsf(charges: Tensor, edge_index: Tensor, r: Tensor, alpha: float, cutoff: float,
                k_e: float = COULOMB_CONSTANT) -> Tensor:
    src, dst = edge_index[0], edge_index[1]
    erfc_rc = math.erfc(alpha * cutoff)
    shift = erfc_rc / cutoff
    slope = erfc_rc / cutoff ** 2 + 2.0 * alpha / math.sqrt(math.pi) * math.exp(-(alpha * cutoff) ** 2) / cutoff
    phi = torch.erfc(alpha * r) / r - shift + (r - cutoff) * slope
    phi = torch.where(r < cutoff, phi, torch.zeros_like(phi))
    node = scatter_sum((0.5 * k_e * charges[src] * charges[dst] * phi).to(torch.float64), dst, charges.shape[0])
    return node + k_e * (-(0.5 * shift + alpha / math.sqrt(math.pi))) * charges.to(torch.float64) ** 2


def ewald_parameters(cutoff: float, accuracy: float) -> Tuple[float, float]:
    root = math.sqrt(-math.log(accuracy))
    alpha = root / cutoff
    return alpha, 2.0 * alpha * root


def reciprocal_lattice(cell: Tensor, k_cutoff: float) -> Tuple[Tensor, Tensor, Tensor]:
    """Integer triples, vectors and squared norms of every ``k != 0`` with ``|k| <= k_cutoff``
    (both ``k`` and ``-k``)."""
    recip = 2.0 * math.pi * torch.linalg.inv(cell).t()
    bounds = torch.ceil(k_cutoff * torch.linalg.norm(cell.detach(), dim=1) / (2.0 * math.pi)).long().tolist()
    axes = [torch.arange(-b, b + 1, device=cell.device) for b in bounds]
    grid = torch.cartesian_prod(*axes).reshape(-1, 3)
    kvec = grid.to(cell.dtype) @ recip
    k2 = (kvec * kvec).sum(-1)
    keep = (k2 > 0) & (k2 <= k_cutoff * k_cutoff)
    return grid[keep], kvec[keep], k2[keep]


def ewald_real(charges: Tensor, edge_index: Tensor, r: Tensor, alpha: float, cutoff: float) -> Tensor:
    src, dst = edge_index[0], edge_index[1]
    phi = torch.where(r < cutoff, torch.erfc(alpha * r) / r, torch.zeros_like(r))
    return scatter_sum((0.5 * charges[src] * charges[dst] * phi).to(torch.float64), dst, charges.shape[0])


def ewald_corrections(charges: Tensor, alpha: float, volume: Tensor) -> Tensor:
    q = charges.to(torch.float64)
    return -(alpha / math.sqrt(math.pi)) * q * q - (math.pi / (2.0 * alpha * alpha)) / volume.to(torch.float64) \
        * q * q.sum()


def ewald_reciprocal(charges: Tensor, pos: Tensor, cell: Tensor, alpha: float, k_cutoff: float,
                     budget: int = RECIPROCAL_BUDGET) -> Tensor:
    q, p, c = charges.to(torch.float64), pos.to(torch.float64), cell.to(torch.float64)
    _, kvec, k2 = reciprocal_lattice(c, k_cutoff)
    weight = 4.0 * math.pi / torch.linalg.det(c).abs() * torch.exp(-0.25 * k2 / (alpha * alpha)) / k2
    step = max(1, budget // max(p.shape[0], 1))
    phi = torch.zeros_like(q)
    for k0 in range(0, kvec.shape[0], step):
        ph = p @ kvec[k0:k0 + step].t()
        cs, sn = torch.cos(ph), torch.sin(ph)
        w = weight[k0:k0 + step]
        phi = phi + cs @ (w * (q @ cs)) + sn @ (w * (q @ sn))
    return 0.5 * q * phi


def coulomb_ewald(charges: Tensor, pos: Tensor, cell: Tensor, edge_index: Tensor, r: Tensor, alpha: float,
                  cutoff: float, k_cutoff: float, k_e: float = COULOMB_CONSTANT) -> Tensor:
    vol = torch.linalg.det(cell.to(torch.float64)).abs()
    return k_e * (ewald_real(charges, edge_index, r, alpha, cutoff) + ewald_reciprocal(charges, pos, cell, alpha, k_cutoff)
                  + ewald_corrections(charges, alpha, vol))


def pme_mesh(cell: Tensor, alpha: float, accuracy: float) -> List[int]:
    factor = 2.0 * alpha / (3.0 * accuracy ** 0.2)
    out = []
    for length in torch.linalg.norm(cell.detach(), dim=1).tolist():
        n = factor * length
        out.append(max(2, 1 << int(math.ceil(math.log(max(n, 1.0)) / math.log(2.0)))))
    return out


def pme_reciprocal(charges: Tensor, pos: Tensor, cell: Tensor, alpha: float, mesh: List[int], order: int) -> Tensor:
    """Per-atom reciprocal shares ``q_i phi_i / 2`` on a smooth-PME mesh (Coulomb units)."""
    from ..ffnn.multipoles import influence, recip_energy, spread
    q = charges.to(torch.float64)
    leaf = q if q.requires_grad else q.detach().requires_grad_(True)
    with torch.enable_grad():
        grid = spread(pos.to(torch.float64), cell.to(torch.float64), leaf, None, None, list(mesh), order)
        e = recip_energy(grid, influence(cell.to(torch.float64), list(mesh), alpha, order, torch.float64, pos.device))
        (phi,) = torch.autograd.grad(e, leaf, create_graph=True)
    return 0.5 * q * phi


def coulomb_pme(charges: Tensor, pos: Tensor, cell: Tensor, edge_index: Tensor, r: Tensor, alpha: float,
                cutoff: float, accuracy: float, order: int, k_e: float = COULOMB_CONSTANT) -> Tensor:
    c = cell.to(torch.float64)
    mesh = pme_mesh(c, alpha, accuracy)
    return k_e * (ewald_real(charges, edge_index, r, alpha, cutoff) + pme_reciprocal(charges, pos, c, alpha, mesh, order)
                  + ewald_corrections(charges, alpha, torch.linalg.det(c).abs()))
