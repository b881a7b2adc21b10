"""3D steerable CNN (Weiler et al., NeurIPS 2018) on the atom-density voxel grid: rotation-
equivariant convolutions whose kernels are expanded in an analytic steerable basis
``K^{l_out l_in}_{m,J} = C^{l_out l_in J} Y^J(x) exp(-(|x| - m)^2 / 2 s^2)`` (Gaussian radial shells
``m = 0, 1, ...`` with per-shell bandlimits ``J <= J_max(m)``), gated non-linearities (scalars
activated, higher fields scaled by sigmoid gates), optional field-wise batch norm, anti-aliased
strides, global average pooling of the final scalars and the shared voxel readout.

The basis construction (bandlimit presets, normalisation of each basis kernel, the
``sqrt((2 l_out + 1) / (n_b * total_in))`` scaling), the field layout and the parameter names follow
the reference (``src/xnn/cnn/models/steerable.py``) so state dicts transplant. On a GPU the convolution
runs as one cuDNN conv3d with the assembled kernel (channels-last conv3d is the library op the
reference also calls).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..nn.blocks import make_activation
from ..o3 import spherical_harmonics, wigner_3j
from .cnn3d import VoxelPotential, default_fields, default_strides, field_dim, global_average_pool, low_pass_filter
from .registry import register_model

BANDLIMITS: Dict[str, Tuple[int, ...]] = {
    "conservative": (0, 2, 4, 6, 8, 10, 12, 14),
    "compromise": (0, 3, 5, 7, 9, 11, 13, 15),
    "sfcnn": (0, 4, 6, 8, 10, 12, 14, 16),
}


def grid_coordinates(size: int, dtype=torch.float64, device=None) -> Tensor:
    """``(size, size, size, 3)`` voxel coordinates with the origin at the centre."""
    c = torch.arange(size, dtype=dtype, device=device) - (size - 1) / 2.0
    return torch.stack(torch.meshgrid(c, c, c, indexing="ij"), -1)


def shell_bandlimits(size: int, bandlimit="compromise") -> Tuple[List[float], List[int]]:
    n = size // 2 + 1
    if isinstance(bandlimit, str):
        if bandlimit not in BANDLIMITS:
            raise ValueError(f"unknown bandlimit {bandlimit!r}; choose one of {sorted(BANDLIMITS)}")
        limits = BANDLIMITS[bandlimit]
    else:
        limits = tuple(int(j) for j in bandlimit)
    if len(limits) < n:
        raise ValueError(f"need a bandlimit for each of the {n} shells, got {len(limits)}")
    return [float(m) for m in range(n)], list(limits[:n])


def angular_kernel_basis(l_in: int, l_out: int, J: int, points: Tensor) -> Tensor:
    """``(2 l_out + 1, 2 l_in + 1, *grid)`` angular block ``sum_M C_{ik M} Y^J_M(x / |x|)`` (zero at the
    origin for ``J > 0``)."""
    if not abs(l_in - l_out) <= J <= l_in + l_out:
        raise ValueError(f"J={J} is not coupled by l_in={l_in}, l_out={l_out}")
    pts = points.to(torch.float64).reshape(-1, 3)
    norm = torch.linalg.norm(pts, dim=-1)
    unit = torch.where(norm[:, None] > 0, pts / norm.clamp(min=1e-300)[:, None], pts)
    Y = spherical_harmonics(J, unit, normalize=False, normalization="component")
    if J > 0:
        Y = torch.where(norm[:, None] > 0, Y, torch.zeros_like(Y))
    block = torch.einsum("ikM,pM->ikp", wigner_3j(l_out, l_in, J, dtype=torch.float64), Y)
    return block.reshape(2 * l_out + 1, 2 * l_in + 1, *points.shape[:-1])


def steerable_kernel_basis(l_in: int, l_out: int, size: int, bandlimit="compromise",
                           shell_width: float = 0.6) -> Optional[Tensor]:
    """The unit-norm basis kernels ``(n_b, 2 l_out + 1, 2 l_in + 1, s, s, s)`` (``None`` if none)."""
    pts = grid_coordinates(size)
    radius = torch.linalg.norm(pts, dim=-1)
    radii, limits = shell_bandlimits(size, bandlimit)
    angular = {J: angular_kernel_basis(l_in, l_out, J, pts) for J in range(abs(l_in - l_out), l_in + l_out + 1)}
    basis = []
    for m, j_max in zip(radii, limits):
        window = torch.exp(-0.5 * ((radius - m) / shell_width) ** 2)
        for J, block in angular.items():
            if J <= j_max:
                k = block * window
                basis.append(k / k.norm())
    return torch.stack(basis) if basis else None


def field_slices(fields: Sequence[int]) -> List[Tuple[int, int, int]]:
    out, start = [], 0
    for l, m in enumerate(fields):
        if m > 0:
            out.append((l, start, start + m * (2 * l + 1)))
            start += m * (2 * l + 1)
    return out


class SteerableConv3d(nn.Module):
    """Equivariant conv3d between field types ``(m_0, m_1, ...)`` (plus ``n_gates`` scalar gate
    outputs): weights ``(m_out, m_in, n_basis)`` per block of orders."""

    def __init__(self, fields_in: Sequence[int], fields_out: Sequence[int], kernel_size: int = 5, n_gates: int = 0,
                 stride: int = 1, padding: Optional[int] = None, dilation: int = 1, bandlimit="compromise",
                 shell_width: float = 0.6):
        super().__init__()
        self.fields_in, self.fields_out = tuple(int(m) for m in fields_in), tuple(int(m) for m in fields_out)
        self.n_gates, self.kernel_size = int(n_gates), int(kernel_size)
        self.stride, self.dilation = int(stride), int(dilation)
        self.padding = self.kernel_size // 2 if padding is None else int(padding)
        self.blocks_in = [(m, l) for l, m in enumerate(self.fields_in) if m > 0]
        self.blocks_out = [(m, l) for l, m in enumerate(self.fields_out) if m > 0]
        if self.n_gates > 0:
            self.blocks_out.append((self.n_gates, 0))
        total_in = sum(m for m, _ in self.blocks_in)
        self.weight = nn.ParameterDict()
        self._basis_keys = []
        for i, (m_out, l_out) in enumerate(self.blocks_out):
            for j, (m_in, l_in) in enumerate(self.blocks_in):
                basis = steerable_kernel_basis(l_in, l_out, self.kernel_size, bandlimit, shell_width)
                if basis is None:
                    self._basis_keys.append((i, j, None))
                    continue
                n_b = basis.shape[0]
                name = f"basis_{i}_{j}"
                self.register_buffer(name, (basis * math.sqrt((2 * l_out + 1) / (n_b * total_in))).to(torch.get_default_dtype()))
                self.weight[f"{i}_{j}"] = nn.Parameter(torch.randn(m_out, m_in, n_b))
                self._basis_keys.append((i, j, name))
        if len(self.weight) == 0:
            raise ValueError("no basis kernel couples these fields at this kernel size and bandlimit")

    def kernel(self) -> Tensor:
        s, rows = self.kernel_size, []
        for i, (m_out, l_out) in enumerate(self.blocks_out):
            cols = []
            for j, (m_in, l_in) in enumerate(self.blocks_in):
                name = self._basis_keys[i * len(self.blocks_in) + j][2]
                d_out, d_in = m_out * (2 * l_out + 1), m_in * (2 * l_in + 1)
                if name is None:
                    ref = next(iter(self.weight.values()))
                    cols.append(ref.new_zeros(d_out, d_in, s, s, s))
                else:
                    cols.append(torch.einsum("uvb,bikxyz->uivkxyz", self.weight[f"{i}_{j}"], getattr(self, name))
                                .reshape(d_out, d_in, s, s, s))
            rows.append(torch.cat(cols, 1))
        return torch.cat(rows, 0)

    def forward(self, x: Tensor) -> Tensor:
        return F.conv3d(x, self.kernel(), stride=self.stride, padding=self.padding, dilation=self.dilation)


class SteerableBatchNorm(nn.Module):
    """Field-wise batch norm: scalars centred; each field divided by the RMS of its norm."""

    def __init__(self, fields: Sequence[int], eps: float = 1e-5, momentum: float = 0.1, affine: bool = True):
        super().__init__()
        self.fields = tuple(int(m) for m in fields)
        self.eps, self.momentum, self.affine = float(eps), float(momentum), bool(affine)
        n_scalar, n_fields = (self.fields[0] if self.fields else 0), sum(self.fields)
        self.register_buffer("running_mean", torch.zeros(n_scalar))
        self.register_buffer("running_var", torch.ones(n_fields))
        if affine:
            self.weight = nn.Parameter(torch.ones(n_fields))
            self.bias = nn.Parameter(torch.zeros(n_scalar))
        else:
            self.register_parameter("weight", None)
            self.register_parameter("bias", None)

    def forward(self, x: Tensor) -> Tensor:
        b, pieces, f0, new_var = x.shape[0], [], 0, []
        for l, start, stop in field_slices(self.fields):
            dim = 2 * l + 1
            m = (stop - start) // dim
            f = x[:, start:stop].reshape(b, m, dim, -1)
            if l == 0:
                if self.training:
                    mean = f.mean(dim=(0, 2, 3))
                    with torch.no_grad():
                        self.running_mean.lerp_(mean, self.momentum)
                else:
                    mean = self.running_mean
                f = f - mean.view(1, m, 1, 1)
            if self.training:
                var = f.pow(2).sum(2).mean(dim=(0, 2))
                new_var.append(var.detach())
            else:
                var = self.running_var[f0:f0 + m]
            f = f / torch.sqrt(var + self.eps).view(1, m, 1, 1)
            if self.affine:
                f = f * self.weight[f0:f0 + m].view(1, m, 1, 1)
                if l == 0:
                    f = f + self.bias.view(1, m, 1, 1)
            pieces.append(f.reshape(b, stop - start, *x.shape[2:]))
            f0 += m
        if self.training and new_var:
            with torch.no_grad():
                self.running_var.lerp_(torch.cat(new_var), self.momentum)
        return torch.cat(pieces, 1)


class GatedBlock(nn.Module):
    def __init__(self, fields_in: Sequence[int], fields_out: Sequence[int], kernel_size: int = 5, stride: int = 1,
                 padding: Optional[int] = None, activation: Optional[str] = "relu",
                 gate_activation: Optional[str] = "sigmoid", normalization: Optional[str] = None,
                 smooth_stride: bool = True, bias: bool = True, bandlimit="compromise", shell_width: float = 0.6):
        super().__init__()
        if normalization not in (None, "batch"):
            raise ValueError(f"normalization must be None or 'batch', got {normalization!r}")
        self.fields_in, self.fields_out = tuple(int(m) for m in fields_in), tuple(int(m) for m in fields_out)
        self.n_scalar = self.fields_out[0] if self.fields_out else 0
        self.n_gates = sum(self.fields_out[1:]) if gate_activation is not None else 0
        self.smooth_stride, self.stride = bool(smooth_stride) and stride > 1, int(stride)
        self.norm = SteerableBatchNorm(self.fields_in) if normalization == "batch" else None
        self.conv = SteerableConv3d(self.fields_in, self.fields_out, kernel_size, self.n_gates,
                                    stride=1 if self.smooth_stride else self.stride, padding=padding,
                                    bandlimit=bandlimit, shell_width=shell_width)
        self.act = make_activation(activation) if activation is not None else None
        self.gate_act = make_activation(gate_activation) if gate_activation is not None else None
        n_bias = (self.n_scalar if self.act is not None else 0) + self.n_gates
        self.bias = nn.Parameter(torch.zeros(n_bias)) if bias and n_bias > 0 else None

    @property
    def out_channels(self) -> int:
        return field_dim(self.fields_out)

    def forward(self, x: Tensor) -> Tensor:
        if self.norm is not None:
            x = self.norm(x)
        y = self.conv(x)
        n_out, b0 = self.out_channels, 0
        scalars = y[:, :self.n_scalar]
        if self.act is not None and self.n_scalar > 0:
            if self.bias is not None:
                scalars = scalars + self.bias[:self.n_scalar].view(1, -1, 1, 1, 1)
                b0 = self.n_scalar
            scalars = self.act(scalars)
        pieces = [scalars]
        if self.n_gates > 0:
            gates = y[:, n_out:]
            if self.bias is not None:
                gates = gates + self.bias[b0:b0 + self.n_gates].view(1, -1, 1, 1, 1)
            gates = self.gate_act(gates)
            g0 = 0
            for l, start, stop in field_slices(self.fields_out):
                if l == 0:
                    continue
                m = (stop - start) // (2 * l + 1)
                field = y[:, start:stop].reshape(y.shape[0], m, 2 * l + 1, *y.shape[2:])
                pieces.append((field * gates[:, g0:g0 + m].unsqueeze(2)).reshape(y.shape[0], stop - start, *y.shape[2:]))
                g0 += m
        else:
            pieces.append(y[:, self.n_scalar:n_out])
        z = torch.cat(pieces, 1)
        return low_pass_filter(z, self.stride, self.stride) if self.smooth_stride else z


@register_model("se3cnn")
class SteerableCNN(VoxelPotential):
    def __init__(self, species: Sequence[int] = (1, 6, 8), cutoff: float = 4.0, grid_size: int = 17,
                 fields: Optional[Sequence[Sequence[int]]] = None, n_features: int = 32, n_blocks: int = 3,
                 l_max: int = 2, kernel_size: int = 5, strides: Optional[Sequence[int]] = None,
                 padding: Optional[int] = None, activation: str = "ssp", gate_activation: str = "sigmoid",
                 normalization: Optional[str] = None, smooth_stride: bool = True, bandlimit="compromise",
                 shell_width: float = 0.6, sigma: Optional[float] = None, cutoff_fn: Optional[str] = "cosine",
                 include_center: bool = True, readout_activation: str = "ssp", energy_shift: float = 0.0,
                 energy_scale: float = 1.0, atomic_energies=None):
        fields = [tuple(int(m) for m in f) for f in (fields or default_fields(n_features, n_blocks, l_max))]
        if not fields or any(m > 0 for m in fields[-1][1:]) or fields[-1][0] < 1:
            raise ValueError("the last block must output scalar fields only")
        strides = list(strides) if strides is not None else default_strides(len(fields))
        if len(strides) != len(fields):
            raise ValueError("strides must have one entry per block")
        super().__init__(species, cutoff, grid_size, fields[-1][0], sigma, cutoff_fn, include_center,
                         readout_activation, energy_shift, energy_scale, atomic_energies)
        self.fields = fields
        blocks, f_in = [], (self.n_channels,)
        for f_out, stride in zip(fields, strides):
            blocks.append(GatedBlock(f_in, f_out, kernel_size, stride, padding, activation, gate_activation,
                                     normalization, smooth_stride, True, bandlimit, shell_width))
            f_in = f_out
        self.blocks = nn.Sequential(*blocks)

    def trunk(self, grid: Tensor) -> Tensor:
        return global_average_pool(self.blocks(grid))

    @classmethod
    def from_config(cls, cfg) -> "SteerableCNN":
        e = dict(cfg.extra or {})
        opts = cls._common_config_options(cfg)
        bl = e.get("bandlimit", "compromise")
        return cls(fields=None if e.get("fields") is None else [[int(m) for m in f] for f in e["fields"]],
                   n_features=cfg.n_features, n_blocks=cfg.n_interactions, l_max=int(e.get("l_max", 2)),
                   kernel_size=int(e.get("kernel_size", 5)),
                   strides=None if e.get("strides") is None else [int(s) for s in e["strides"]],
                   padding=None if e.get("padding") is None else int(e["padding"]),
                   activation=e.get("activation", "ssp"), gate_activation=e.get("gate_activation", "sigmoid"),
                   normalization=e.get("normalization"), smooth_stride=bool(e.get("smooth_stride", True)),
                   bandlimit=bl if isinstance(bl, str) else [int(j) for j in bl],
                   shell_width=float(e.get("shell_width", 0.6)), **opts)
