"""Element-aware warps of the interatomic distance applied before the radial basis.

Foundation MACE models (MACE-MP-0 and relatives) expand a *transformed* distance in their
Bessel basis: each edge's length is measured in units of a radius built from the covalent
radii of its two elements, so a C-H bond and a Cs-I bond land on comparable coordinates.
Two warps exist, named by the option strings MACE checkpoints store:

* ``"Agnesi"``: ``T(r) = 1 / (1 + a u^q / (1 + u^(q - p)))`` with ``u = r / r0`` and ``r0`` the
  mean covalent radius of the pair (the radial transformation of ACEpotentials.jl,
  J. Chem. Phys. 159, 164101 (2023); constants a = 1.0805, q = 0.9183, p = 4.5791 as
  published for MACE-MP-0, arXiv:2401.00096);
* ``"Soft"``: a tanh switch from a floor ``3/4 r0`` to the identity, centred between ``3/4 r0``
  and ``4/3 r0`` with ``r0`` the *sum* of the covalent radii and steepness ``alpha / width``.

The covalent radii are Cordero et al., Dalton Trans. 2832 (2008), indexed by atomic number,
0.2 A for elements without a value. Constants and table are buffers, so checkpoints carry them.

Parity: ``src/xnn/gnn/featurizers/radial.py:41-164`` of the reference (same registry keys).
"""
from __future__ import annotations

from typing import Dict

import torch
from torch import Tensor, nn

from ..data.elements import COVALENT_RADII

_N_Z = 119          # atomic numbers 0..118


def _radii_table() -> Tensor:
    vals = list(COVALENT_RADII) + [0.2] * (_N_Z - len(COVALENT_RADII))
    return torch.tensor(vals[:_N_Z], dtype=torch.float64)


class _PairRadiusWarp(nn.Module):
    """Common part: the covalent radii of both ends of every edge."""

    def __init__(self):
        super().__init__()
        self.register_buffer("covalent_radii", _radii_table())

    def _ends(self, r: Tensor, atomic_numbers: Tensor, edge_index: Tensor):
        rc = self.covalent_radii.to(r.dtype)[atomic_numbers]
        return rc[edge_index[0]], rc[edge_index[1]]


class IdentityDistanceTransform(nn.Module):
    """No warp: ``T(r) = r`` (the ``"None"`` option)."""

    def forward(self, r: Tensor, atomic_numbers: Tensor, edge_index: Tensor) -> Tensor:
        return r


class AgnesiDistanceTransform(_PairRadiusWarp):
    def __init__(self, a: float = 1.0805, q: float = 0.9183, p: float = 4.5791):
        super().__init__()
        self.register_buffer("a", torch.tensor(float(a), dtype=torch.float64))
        self.register_buffer("q", torch.tensor(float(q), dtype=torch.float64))
        self.register_buffer("p", torch.tensor(float(p), dtype=torch.float64))

    def forward(self, r: Tensor, atomic_numbers: Tensor, edge_index: Tensor) -> Tensor:
        ri, rj = self._ends(r, atomic_numbers, edge_index)
        u = 2.0 * r / (ri + rj)
        a, q, p = (t.to(r.dtype) for t in (self.a, self.q, self.p))
        return torch.reciprocal(1.0 + a * torch.pow(u, q) / (1.0 + torch.pow(u, q - p)))


class SoftDistanceTransform(_PairRadiusWarp):
    def __init__(self, alpha: float = 4.0):
        super().__init__()
        self.register_buffer("alpha", torch.tensor(float(alpha), dtype=torch.float64))

    def forward(self, r: Tensor, atomic_numbers: Tensor, edge_index: Tensor) -> Tensor:
        ri, rj = self._ends(r, atomic_numbers, edge_index)
        s = ri + rj
        lo, hi = 0.75 * s, s * (4.0 / 3.0)
        w = 0.5 * (1.0 + torch.tanh(self.alpha.to(r.dtype) * (r - 0.5 * (lo + hi)) / (hi - lo)))
        return lo + w * (r - lo)


DISTANCE_TRANSFORMS: Dict[object, type] = {
    None: IdentityDistanceTransform,
    "None": IdentityDistanceTransform,
    "Agnesi": AgnesiDistanceTransform,
    "Soft": SoftDistanceTransform,
}
