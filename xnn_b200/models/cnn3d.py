"""Voxel-grid potentials: per-atom density cubes through a 3D CNN to atomic energies.

:class:`VoxelPotential` holds the featurizer, the readout MLP (zero-initialised last layer), the
energy scale / shift and per-element reference energies; :class:`CNN3D` is a stack of
``Conv3d -> (Gaussian low-pass + stride) -> [BatchNorm] -> activation`` blocks followed by global
average pooling. Strided blocks blur with a separable Gaussian (``sigma = 0.5 sqrt(s^2 - 1)``)
before subsampling. Channel defaults, options and parameter names follow the reference
(``src/xnn/cnn/models/base.py``, ``cnn3d.py``).
"""
from __future__ import annotations

from functools import lru_cache
from typing import Optional, Sequence

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..featurizers.voxel import VoxelGrid
from ..nn.blocks import make_activation
from .base import InteratomicPotential
from .registry import register_model

_MAX_Z = 120


def field_dim(fields: Sequence[int]) -> int:
    return int(sum(m * (2 * l + 1) for l, m in enumerate(fields)))


def default_fields(n_features: int, n_blocks: int, l_max: int = 2) -> list:
    if n_blocks < 1:
        raise ValueError("n_blocks must be at least 1")
    out = []
    for t in range(n_blocks - 1):
        m0 = max(1, n_features // 4) * 2 ** t
        out.append(tuple(max(1, m0 >> l) for l in range(l_max + 1)))
    out.append((int(n_features),))
    return out


def default_strides(n_blocks: int) -> list:
    return [1 if t in (0, n_blocks - 1) else 2 for t in range(n_blocks)]


@lru_cache(maxsize=64)
def _blur_matrix(sigma: float, size: int, n: int, stride: int, dtype, device) -> Tensor:
    r = torch.arange(size, dtype=torch.float64) - size // 2
    taps = torch.exp(-r ** 2 / (2 * sigma ** 2))
    taps = taps / taps.sum()
    n_out = (n - 1) // stride + 1
    rows = torch.arange(n_out)
    m = torch.zeros(n_out, n, dtype=torch.float64)
    for k in range(size):
        cols = rows * stride - size // 2 + k
        ok = (cols >= 0) & (cols < n)
        m[rows[ok], cols[ok]] = taps[k]
    return m.to(device=device, dtype=dtype)


def low_pass_filter(x: Tensor, scale: float, stride: int = 1) -> Tensor:
    """Separable Gaussian blur of the last three axes (zero padding), subsampled by ``stride``."""
    if scale <= 1:
        if stride != 1:
            raise ValueError("a stride needs a low-pass scale larger than one")
        return x
    sigma = 0.5 * (scale ** 2 - 1) ** 0.5
    size = int(1 + 2 * 2.5 * sigma)
    size += 1 - size % 2
    lead, (nx, ny, nz) = x.shape[:-3], x.shape[-3:]
    mx, my, mz = (_blur_matrix(sigma, size, n, stride, x.dtype, x.device) for n in (nx, ny, nz))
    x = my @ (x @ mz.t())
    x = mx @ x.reshape(*lead, nx, -1)
    return x.view(*lead, mx.shape[0], my.shape[0], mz.shape[0])


def global_average_pool(x: Tensor) -> Tensor:
    return x.flatten(2).mean(-1)


class VoxelPotential(InteratomicPotential):
    head_modules = ("readout", "energy_scale", "energy_shift", "atom_ref")

    def __init__(self, species=(1, 6, 8), cutoff: float = 4.0, grid_size: int = 17, n_features: int = 32,
                 sigma: Optional[float] = None, cutoff_fn: Optional[str] = "cosine", include_center: bool = True,
                 readout_activation: str = "ssp", energy_shift: float = 0.0, energy_scale: float = 1.0,
                 atomic_energies=None, featurizer: Optional[nn.Module] = None):
        super().__init__()
        self.species = [int(z) for z in species]
        self.cutoff = float(cutoff)
        self.node_feature_dim = int(n_features)
        self.featurizer = featurizer if featurizer is not None else VoxelGrid(self.species, cutoff, grid_size, sigma,
                                                                              cutoff_fn, include_center)
        h = max(1, n_features // 2)
        self.readout = nn.Sequential(nn.Linear(n_features, h), make_activation(readout_activation), nn.Linear(h, 1))
        nn.init.zeros_(self.readout[-1].weight)
        nn.init.zeros_(self.readout[-1].bias)
        self.register_buffer("energy_scale", torch.tensor(float(energy_scale)))
        self.register_buffer("energy_shift", torch.tensor(float(energy_shift)))
        self.atom_ref = nn.Embedding(_MAX_Z, 1)
        nn.init.zeros_(self.atom_ref.weight)
        if atomic_energies is not None:
            self.set_atomic_energies(atomic_energies)

    @property
    def grid_size(self) -> int:
        return self.featurizer.grid_size

    @property
    def n_channels(self) -> int:
        return self.featurizer.n_channels

    def receptive_field(self) -> float:
        return self.cutoff

    def set_energy_scale_shift(self, scale: float, shift: float) -> None:
        with torch.no_grad():
            self.energy_scale.fill_(float(scale))
            self.energy_shift.fill_(float(shift))

    def set_atomic_energies(self, values) -> None:
        ae = torch.as_tensor(values, dtype=self.atom_ref.weight.dtype).flatten()
        if ae.numel() != len(self.species):
            raise ValueError(f"got {ae.numel()} atomic energies for {len(self.species)} species")
        with torch.no_grad():
            self.atom_ref.weight[torch.tensor(self.species), 0] = ae

    def trunk(self, grid: Tensor) -> Tensor:
        raise NotImplementedError

    def node_features_energy_grid(self, grid: Tensor, z: Tensor):
        f = self.trunk(grid)
        return f, self.energy_scale * self.readout(f).squeeze(-1) + self.energy_shift + self.atom_ref(z).squeeze(-1)

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        return self.node_features_energy_grid(self.featurizer.voxelize(atomic_numbers, edge_index, edge_vec),
                                              atomic_numbers)

    def forward(self, data: AtomicGraph) -> dict:
        f, e = self.node_features_energy_grid(self.featurizer(data), data.atomic_numbers)
        return {"node_energy": e, "energy": self.aggregate_energy(e, data), "node_features": f}

    @staticmethod
    def _common_config_options(cfg) -> dict:
        e = dict(cfg.extra or {})
        species = [int(z) for z in e.get("species") or [1, 6, 8]]
        sigma = e.get("sigma")
        return dict(species=species, cutoff=cfg.cutoff, grid_size=int(e.get("grid_size", 17)),
                    sigma=None if sigma is None else float(sigma), cutoff_fn=e.get("cutoff_fn", "cosine"),
                    include_center=bool(e.get("include_center", True)),
                    readout_activation=e.get("readout_activation", "ssp"),
                    energy_shift=float(e.get("energy_shift", 0.0)), energy_scale=float(e.get("energy_scale", 1.0)),
                    atomic_energies=e.get("atomic_energies"))


class Conv3dBlock(nn.Module):
    def __init__(self, c_in: int, c_out: int, kernel_size: int = 5, stride: int = 1, padding: Optional[int] = None,
                 activation: Optional[str] = "relu", normalization: Optional[str] = None, smooth_stride: bool = True):
        super().__init__()
        if normalization not in (None, "batch"):
            raise ValueError(f"normalization must be None or 'batch', got {normalization!r}")
        padding = kernel_size // 2 if padding is None else int(padding)
        self.smooth_stride = bool(smooth_stride) and stride > 1
        self.stride = int(stride)
        self.conv = nn.Conv3d(c_in, c_out, kernel_size, padding=padding, stride=1 if self.smooth_stride else self.stride)
        self.norm = nn.BatchNorm3d(c_out) if normalization == "batch" else None
        self.act = make_activation(activation) if activation is not None else None

    def forward(self, x: Tensor) -> Tensor:
        x = self.conv(x)
        if self.smooth_stride:
            x = low_pass_filter(x, self.stride, self.stride)
        if self.norm is not None:
            x = self.norm(x)
        return self.act(x) if self.act is not None else x


@register_model("cnn3d")
class CNN3D(VoxelPotential):
    def __init__(self, species=(1, 6, 8), cutoff: float = 4.0, grid_size: int = 17, channels=None, n_features: int = 32,
                 n_blocks: int = 3, kernel_size: int = 5, strides=None, padding: Optional[int] = None,
                 activation: str = "ssp", normalization: Optional[str] = None, smooth_stride: bool = True,
                 sigma: Optional[float] = None, cutoff_fn: Optional[str] = "cosine", include_center: bool = True,
                 readout_activation: str = "ssp", energy_shift: float = 0.0, energy_scale: float = 1.0,
                 atomic_energies=None):
        if channels is None:
            channels = [field_dim(f) for f in default_fields(n_features, n_blocks)]
        channels = [int(c) for c in channels]
        strides = default_strides(len(channels)) if strides is None else list(strides)
        if len(strides) != len(channels):
            raise ValueError("strides must have one entry per block")
        super().__init__(species, cutoff, grid_size, channels[-1], sigma, cutoff_fn, include_center,
                         readout_activation, energy_shift, energy_scale, atomic_energies)
        self.channels = channels
        blocks, c_in = [], self.n_channels
        for c_out, s in zip(channels, strides):
            blocks.append(Conv3dBlock(c_in, c_out, kernel_size, s, padding, activation, normalization, smooth_stride))
            c_in = c_out
        self.blocks = nn.Sequential(*blocks)

    def trunk(self, grid: Tensor) -> Tensor:
        return global_average_pool(self.blocks(grid))

    @classmethod
    def from_config(cls, cfg) -> "CNN3D":
        e = dict(cfg.extra or {})
        ch, st, pad = e.get("channels"), e.get("strides"), e.get("padding")
        return cls(channels=None if ch is None else [int(c) for c in ch], n_features=cfg.n_features,
                   n_blocks=cfg.n_interactions, kernel_size=int(e.get("kernel_size", 5)),
                   strides=None if st is None else [int(s) for s in st], padding=None if pad is None else int(pad),
                   activation=e.get("activation", "ssp"), normalization=e.get("normalization"),
                   smooth_stride=bool(e.get("smooth_stride", True)), **cls._common_config_options(cfg))
