"""Per-atom voxel grids of the neighbour density: a ``grid_size^3`` cube of side ``2 cutoff``
centred on every atom, one channel per species, Gaussians of width ``sigma`` (the grid spacing by
default) at the neighbours' relative positions weighted by a cosine envelope, plus the centre
atom's own Gaussian. Separable: each Gaussian is the outer product of three 1D profiles.
Options follow the reference (``src/xnn/cnn/featurizers/voxel.py``)."""
from __future__ import annotations

from typing import Optional, Sequence

import torch
from torch import Tensor, nn

from ..nn.cutoff import CosineCutoff

_MAX_Z = 120
VOXEL_BLOCK = 1 << 24


class VoxelGrid(nn.Module):
    def __init__(self, species: Sequence[int], cutoff: float = 4.0, grid_size: int = 17, sigma: Optional[float] = None,
                 cutoff_fn: Optional[str] = "cosine", include_center: bool = True):
        super().__init__()
        if cutoff_fn not in (None, "cosine"):
            raise ValueError(f"cutoff_fn must be None or 'cosine', got {cutoff_fn!r}")
        if grid_size < 1:
            raise ValueError("grid_size must be positive")
        self.species = [int(z) for z in species]
        if len(set(self.species)) != len(self.species):
            raise ValueError("species must not repeat")
        self.cutoff, self.grid_size = float(cutoff), int(grid_size)
        self.spacing = 2.0 * self.cutoff / self.grid_size
        self.sigma = float(sigma) if sigma is not None else self.spacing
        self.include_center = bool(include_center)
        self.envelope = CosineCutoff(self.cutoff) if cutoff_fn == "cosine" else None
        index = torch.full((_MAX_Z,), -1, dtype=torch.long)
        for c, z in enumerate(self.species):
            index[z] = c
        self.register_buffer("species_index", index)
        k = torch.arange(self.grid_size, dtype=torch.get_default_dtype())
        self.register_buffer("axis", (k - (self.grid_size - 1) / 2.0) * self.spacing)

    @property
    def output_dim(self) -> int:
        return len(self.species)

    @property
    def n_channels(self) -> int:
        return len(self.species)

    def channel_index(self, z: Tensor) -> Tensor:
        idx = self.species_index[z]
        if bool((idx < 0).any()):
            raise ValueError(f"atomic numbers {sorted(set(z[idx < 0].tolist()))} have no density channel "
                             f"(species={self.species})")
        return idx

    def _profile(self, c: Tensor) -> Tensor:
        return torch.exp(-(self.axis.to(c.dtype)[None, :] - c[:, None]) ** 2 / (2.0 * self.sigma ** 2))

    def voxelize(self, z: Tensor, edge_index: Tensor, edge_vec: Tensor) -> Tensor:
        n, nc, s = z.shape[0], self.n_channels, self.grid_size
        ch = self.channel_index(z)
        grid = torch.zeros(n * nc, s, s, s, dtype=edge_vec.dtype, device=edge_vec.device)
        if self.include_center and n:
            g = self._profile(edge_vec.new_zeros(1))[0]
            blob = g[:, None, None] * g[None, :, None] * g[None, None, :]
            grid = grid.index_add(0, torch.arange(n, device=z.device) * nc + ch, blob.expand(n, s, s, s))
        src, dst = edge_index[0], edge_index[1]
        rel = -edge_vec
        w = self.envelope(torch.linalg.norm(rel, dim=-1)) if self.envelope is not None else torch.ones_like(rel[:, 0])
        target = dst * nc + ch[src]
        block = max(1, VOXEL_BLOCK // (s * s * s))
        for e0 in range(0, rel.shape[0], block):
            r = rel[e0:e0 + block]
            gx, gy, gz = self._profile(r[:, 0]), self._profile(r[:, 1]), self._profile(r[:, 2])
            dens = w[e0:e0 + block, None, None, None] * gx[:, :, None, None] * gy[:, None, :, None] * gz[:, None, None, :]
            grid = grid.index_add(0, target[e0:e0 + block], dens)
        return grid.view(n, nc, s, s, s)

    def forward(self, data) -> Tensor:
        return self.voxelize(data.atomic_numbers, data.edge_index, data.edge_vectors())
