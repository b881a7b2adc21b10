"""Element-resolved radial and angular symmetry functions (Behler-Parrinello / ANI).

Radial: ``G_i = pref sum_j exp(-eta (r_ij - Rs)^2) fc(r_ij)`` per ``(eta, Rs)`` and neighbour
species. Angular (ANI form): ``G_i = sum_{j<k} 2 ((1 + cos(theta_ijk - theta_s)) / 2)^zeta
exp(-eta ((r_ij + r_ik)/2 - Rs)^2) fc(r_ij) fc(r_ik)`` per ``(eta, zeta, Rs, theta_s)`` and
unordered neighbour-species pair, with ``theta = acos(cos_factor cos theta)`` (0.95 for ANI keeps
``acos`` away from its singular end points). With ``prefactor=0.25`` and ``cos_factor=0.95``
these are the AEV of torchani. Parameter order, buffers and bucketing follow the reference
(``src/xnn/dnn/featurizers/symmetry_functions.py:44,184``).
"""
from __future__ import annotations

import itertools
from typing import Optional, Tuple

import torch
from torch import Tensor, nn

from ..nn.cutoff import CosineCutoff
from ..ops.scatter import build_center_pairs

_N_Z = 119


class RadialSymmetryFunctions(nn.Module):
    def __init__(self, species, cutoff: float = 6.0, etas=(0.05, 0.5, 2.0, 8.0), rs=(0.0,), prefactor: float = 1.0):
        super().__init__()
        self.species = [int(z) for z in species]
        self.cutoff = float(cutoff)
        self.prefactor = float(prefactor)
        bucket = torch.full((_N_Z,), -1, dtype=torch.long)
        for i, z in enumerate(self.species):
            bucket[z] = i
        self.register_buffer("_bucket", bucket, persistent=False)
        self.register_buffer("etas", torch.tensor([float(e) for e in etas]))
        self.register_buffer("rs", torch.tensor([float(r) for r in rs]))
        self.cutoff_fn = CosineCutoff(cutoff)
        self._n_params = len(etas) * len(rs)

    @property
    def output_dim(self) -> int:
        return self._n_params * len(self.species)

    def edge_terms(self, r: Tensor, weight: Tensor) -> Tensor:
        """``weight * exp(-eta (r - Rs)^2)`` per edge, ``(E, n_eta * n_rs)`` in ``(eta, Rs)`` order."""
        g = torch.exp(-self.etas.view(-1, 1) * (r.view(-1, 1, 1) - self.rs) ** 2)
        return (g * weight.view(-1, 1, 1)).reshape(r.shape[0], self._n_params)

    def forward(self, data) -> Tensor:
        return self.compute(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.num_nodes)

    def compute(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor, num_nodes: int,
                r: Optional[Tensor] = None) -> Tensor:
        if r is None:
            r = torch.linalg.norm(edge_vec, dim=-1)
        src, dst = edge_index[0], edge_index[1]
        bucket = self._bucket[atomic_numbers[src]]
        fc = torch.where(bucket >= 0, self.prefactor * self.cutoff_fn(r), torch.zeros_like(r))
        g = self.edge_terms(r, fc)
        ns = len(self.species)
        out = torch.zeros(num_nodes * ns, self._n_params, device=r.device, dtype=r.dtype)
        return out.index_add_(0, dst * ns + bucket.clamp(min=0), g).reshape(num_nodes, ns * self._n_params)


class AngularSymmetryFunctions(nn.Module):
    def __init__(self, species, cutoff: float = 4.0, etas=(0.5,), zetas=(8.0,), rs=(0.0, 1.5, 3.0),
                 theta_s=(0.0, 1.5708, 3.1416, 4.7124), cos_factor: float = 1.0):
        super().__init__()
        self.species = [int(z) for z in species]
        self.cutoff = float(cutoff)
        self.cos_factor = float(cos_factor)
        self.cutoff_fn = CosineCutoff(cutoff)
        for name, vals in (("etas", etas), ("zetas", zetas), ("rs", rs), ("theta_s", theta_s)):
            self.register_buffer(name, torch.tensor([float(v) for v in vals]))
        grid = list(itertools.product(etas, zetas, rs, theta_s))
        self.register_buffer("grid", torch.tensor(grid, dtype=torch.get_default_dtype()))
        self._n_params = len(grid)
        self.pairs = list(itertools.combinations_with_replacement(self.species, 2))
        bucket = torch.full((_N_Z, _N_Z), -1, dtype=torch.long)
        for i, (a, b) in enumerate(self.pairs):
            bucket[a, b] = bucket[b, a] = i
        self.register_buffer("_bucket", bucket, persistent=False)

    @property
    def output_dim(self) -> int:
        return self._n_params * len(self.pairs)

    def forward(self, data) -> Tensor:
        return self.compute(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.num_nodes)

    def compute(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor, num_nodes: int,
                r: Optional[Tensor] = None, triplets: Optional[Tuple[Tensor, Tensor]] = None) -> Tensor:
        r = torch.linalg.norm(edge_vec, dim=-1) if r is None else r
        if triplets is not None:
            i1, i2 = triplets
        else:
            inside = torch.nonzero(r <= self.cutoff).flatten()
            e1, e2 = build_center_pairs(edge_index[1].index_select(0, inside), num_nodes)
            i1, i2 = inside.index_select(0, e1), inside.index_select(0, e2)
        center = edge_index[1].index_select(0, i1)
        n_pairs = len(self.pairs)
        out = torch.zeros(num_nodes * n_pairs, self._n_params, device=edge_vec.device, dtype=edge_vec.dtype)
        if i1.numel() == 0:
            return out.reshape(num_nodes, n_pairs * self._n_params)
        fc = self.cutoff_fn(r)
        va, vb = edge_vec.index_select(0, i1), edge_vec.index_select(0, i2)
        ra, rb = r.index_select(0, i1), r.index_select(0, i2)
        cos_t = (va * vb).sum(-1) / (ra * rb).clamp(min=1e-10)
        theta = torch.acos((self.cos_factor * cos_t).clamp(-1.0, 1.0))
        ang = (0.5 * (1.0 + torch.cos(theta.view(-1, 1, 1) - self.theta_s))) ** self.zetas.view(-1, 1)
        src = edge_index[0]
        bucket = self._bucket[atomic_numbers[src.index_select(0, i1)], atomic_numbers[src.index_select(0, i2)]]
        w = fc.index_select(0, i1) * fc.index_select(0, i2)
        w = torch.where(bucket >= 0, 2.0 * w, torch.zeros_like(w))
        rad = torch.exp(-self.etas.view(-1, 1) * ((0.5 * (ra + rb)).view(-1, 1, 1) - self.rs) ** 2) * w.view(-1, 1, 1)
        ne, nz, nr, nt = rad.shape[1], ang.shape[1], rad.shape[2], ang.shape[2]
        g = (rad.view(-1, ne, 1, nr, 1) * ang.view(-1, 1, nz, 1, nt)).reshape(-1, self._n_params)
        return out.index_add_(0, center * n_pairs + bucket.clamp(min=0), g).reshape(num_nodes, n_pairs * self._n_params)
