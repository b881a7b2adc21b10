"""Spherical CNN (Cohen et al., ICLR 2018) on per-atom potential maps: every atom sees its neighbours
as a Coulomb-like potential ``sum_j Z_i Z_j / |p - r_ij|^k`` sampled on a sphere of radius ``radius``
(Driscoll-Healy grid, one channel per neighbour species); residual blocks of S2 and SO(3)
correlations computed in the spectral domain (FFT along the Euler angles, Wigner-d along beta,
Driscoll-Healy quadrature), batch norm, the SO(3) integral of the last features, and the voxel
readout (or a deep-set readout per structure).

Grids, quadrature, transforms, filter bases (near-identity and equatorial), normalisations, the
block schedule of the paper (Table 3) and the parameter names follow the reference
(``src/xnn/cnn/models/spherical.py``, ``cnn/featurizers/spherical.py``). The spectral products run
as complex einsums (batched cuBLAS/cuFFT on a GPU).
"""
from __future__ import annotations

import math
from functools import lru_cache
from typing import Dict, Optional, Sequence, Tuple

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn import CosineCutoff
from ..nn.blocks import make_activation
from .cnn3d import VoxelPotential
from .registry import register_model

_MAX_Z = 120
POINT_BLOCK = 1 << 22


def so3_betas(b: int, dtype=torch.float64) -> Tensor:
    return (torch.arange(2 * b, dtype=dtype) + 0.5) * math.pi / (2 * b)


def so3_alphas(b: int, dtype=torch.float64) -> Tensor:
    return torch.arange(2 * b, dtype=dtype) * (2 * math.pi / (2 * b))


def s2_grid_points(b: int, dtype=torch.float64) -> Tensor:
    """``(2b, 2b, 3)`` unit vectors of the Driscoll-Healy grid (beta rows, alpha columns)."""
    bb, aa = torch.meshgrid(so3_betas(b, dtype), so3_alphas(b, dtype), indexing="ij")
    return torch.stack([torch.sin(bb) * torch.cos(aa), torch.sin(bb) * torch.sin(aa), torch.cos(bb)], -1)


@lru_cache(maxsize=None)
def quadrature_weights(b: int) -> Tensor:
    """Driscoll-Healy weights of the ``2b`` beta samples (normalised for the SO(3) grid)."""
    beta = so3_betas(b)
    k = torch.arange(b, dtype=torch.float64)
    series = (torch.sin((2 * k + 1)[None] * beta[:, None]) / (2 * k + 1)[None]).sum(1)
    return (2.0 / b) * torch.sin(beta) * series / (2.0 * (2 * b) ** 2)


@lru_cache(maxsize=None)
def _spin_y(l: int):
    m = torch.arange(-l, l + 1, dtype=torch.float64)
    jp = torch.zeros(2 * l + 1, 2 * l + 1, dtype=torch.complex128)
    jp[torch.arange(1, 2 * l + 1), torch.arange(0, 2 * l)] = torch.sqrt(l * (l + 1) - m[:-1] * (m[:-1] + 1)).to(torch.complex128)
    ev, vec = torch.linalg.eigh((jp - jp.conj().T) / 2j)
    return ev.round(), vec


def wigner_d(l: int, beta: Tensor) -> Tensor:
    """Real small Wigner ``d^l(beta)`` ``(..., 2l+1, 2l+1)`` as ``exp(-i beta J_y)`` from the
    eigenbasis of ``J_y`` (rows and columns ``m = -l..l``)."""
    ev, vec = _spin_y(l)
    beta = torch.as_tensor(beta, dtype=torch.float64)
    return torch.einsum("mk,...k,nk->...mn", vec, torch.exp(-1j * beta[..., None] * ev), vec.conj()).real


@lru_cache(maxsize=None)
def wigner_d_table(b_grid: int, b_spec: int) -> Tensor:
    """``(2 b_grid, b_spec, 2 b_spec - 1, 2 b_spec - 1)``: ``d^l`` at every grid beta, centred."""
    t = torch.zeros(2 * b_grid, b_spec, 2 * b_spec - 1, 2 * b_spec - 1, dtype=torch.float64)
    betas = so3_betas(b_grid)
    for l in range(b_spec):
        o = b_spec - 1 - l
        t[:, l, o:o + 2 * l + 1, o:o + 2 * l + 1] = wigner_d(l, betas)
    return t


def _band(x: Tensor, b: int, dim: int) -> Tensor:
    n = x.shape[dim]
    return torch.cat([x.narrow(dim, n - (b - 1), b - 1), x.narrow(dim, 0, b)], dim)


def _unband(x: Tensor, size: int, dim: int) -> Tensor:
    b = (x.shape[dim] + 1) // 2
    shape = list(x.shape)
    shape[dim] = size - (2 * b - 1)
    return torch.cat([x.narrow(dim, b - 1, b), x.new_zeros(shape), x.narrow(dim, 0, b - 1)], dim)


class S2Transform(nn.Module):
    """Forward / inverse spherical-harmonic transform of ``(..., 2b, 2b)`` grids."""

    def __init__(self, b_grid: int, b_spec: int):
        super().__init__()
        if b_spec > b_grid:
            raise ValueError(f"the spectrum bandwidth {b_spec} exceeds the grid bandwidth {b_grid}")
        self.b_grid, self.b_spec = int(b_grid), int(b_spec)
        dt = torch.get_default_dtype()
        self.register_buffer("d", wigner_d_table(b_grid, b_spec)[:, :, :, b_spec - 1].to(dt))
        self.register_buffer("weights", (quadrature_weights(b_grid) * (2 * b_grid)).to(dt))
        self.register_buffer("degree", (2 * torch.arange(b_spec) + 1).to(dt))
        self.register_buffer("m_index", torch.remainder(torch.arange(-(b_spec - 1), b_spec), 2 * b_grid))
        self.register_buffer("d_weighted", self.d * self.weights[:, None, None], persistent=False)
        self.register_buffer("d_degree", self.d * self.degree[None, :, None], persistent=False)

    def analyze(self, x: Tensor) -> Tensor:
        spec = _band(torch.fft.fft(x, dim=-1), self.b_spec, -1)
        return torch.einsum("...jm,jlm->...lm", spec, self.d_weighted.to(spec.dtype))

    def synthesize(self, f_hat: Tensor, real: bool = True) -> Tensor:
        rows = torch.einsum("...lm,jlm->...jm", f_hat, self.d_degree.to(f_hat.dtype))
        out = torch.fft.ifft(_unband(rows, 2 * self.b_grid, -1), dim=-1) * (2 * self.b_grid)
        return out.real if real else out


class SO3Transform(nn.Module):
    """Forward / inverse SO(3) Fourier transform of ``(..., 2b, 2b, 2b)`` grids (beta, alpha, gamma)."""

    def __init__(self, b_grid: int, b_spec: int):
        super().__init__()
        if b_spec > b_grid:
            raise ValueError(f"the spectrum bandwidth {b_spec} exceeds the grid bandwidth {b_grid}")
        self.b_grid, self.b_spec = int(b_grid), int(b_spec)
        dt = torch.get_default_dtype()
        self.register_buffer("d", wigner_d_table(b_grid, b_spec).to(dt))
        self.register_buffer("weights", quadrature_weights(b_grid).to(dt))
        self.register_buffer("degree", (2 * torch.arange(b_spec) + 1).to(dt))
        self.register_buffer("m_index", torch.remainder(torch.arange(-(b_spec - 1), b_spec), 2 * b_grid))
        self.register_buffer("d_weighted", self.d * self.weights[:, None, None, None], persistent=False)
        self.register_buffer("d_degree", self.d * self.degree[None, :, None, None], persistent=False)

    def analyze(self, x: Tensor) -> Tensor:
        spec = _band(_band(torch.fft.fft2(x, dim=(-2, -1)), self.b_spec, -2), self.b_spec, -1)
        return torch.einsum("...jmn,jlmn->...lmn", spec, self.d_weighted.to(spec.dtype))

    def synthesize(self, f_hat: Tensor, real: bool = True) -> Tensor:
        rows = torch.einsum("...lmn,jlmn->...jmn", f_hat, self.d_degree.to(f_hat.dtype))
        size = 2 * self.b_grid
        out = torch.fft.ifft2(_unband(_unband(rows, size, -2), size, -1), dim=(-2, -1)) * size ** 2
        return out.real if real else out


def so3_integrate(x: Tensor) -> Tensor:
    w = quadrature_weights(x.shape[-1] // 2).to(device=x.device, dtype=x.dtype)
    return torch.einsum("...jkl,j->...", x, w)


def s2_near_identity_grid(max_beta: float = math.pi / 8, n_alpha: int = 8, n_beta: int = 3) -> Tensor:
    beta = torch.arange(1, n_beta + 1, dtype=torch.float64) * max_beta / n_beta
    alpha = torch.arange(n_alpha, dtype=torch.float64) * (2 * math.pi / n_alpha)
    bb, aa = torch.meshgrid(beta, alpha, indexing="ij")
    return torch.stack([bb.flatten(), aa.flatten()], 1)


def s2_equatorial_grid(max_beta: float = 0.0, n_alpha: int = 32, n_beta: int = 1) -> Tensor:
    beta = torch.linspace(math.pi / 2 - max_beta, math.pi / 2 + max_beta, n_beta, dtype=torch.float64)
    alpha = torch.arange(n_alpha, dtype=torch.float64) * (2 * math.pi / n_alpha)
    bb, aa = torch.meshgrid(beta, alpha, indexing="ij")
    return torch.stack([bb.flatten(), aa.flatten()], 1)


def so3_near_identity_grid(max_beta: float = math.pi / 8, max_gamma: float = 2 * math.pi, n_alpha: int = 8,
                           n_beta: int = 3, n_gamma: Optional[int] = None) -> Tensor:
    n_gamma = n_alpha if n_gamma is None else n_gamma
    beta = torch.arange(1, n_beta + 1, dtype=torch.float64) * max_beta / n_beta
    alpha = torch.arange(n_alpha, dtype=torch.float64) * (2 * math.pi / n_alpha)
    pre = torch.linspace(-max_gamma, max_gamma, n_gamma, dtype=torch.float64)
    bb, aa, cc = torch.meshgrid(beta, alpha, pre, indexing="ij")
    return torch.stack([bb.flatten(), aa.flatten(), (cc - aa).flatten()], 1)


def so3_equatorial_grid(max_beta: float = 0.0, max_gamma: float = math.pi / 8, n_alpha: int = 32, n_beta: int = 1,
                        n_gamma: int = 2) -> Tensor:
    beta = torch.linspace(math.pi / 2 - max_beta, math.pi / 2 + max_beta, n_beta, dtype=torch.float64)
    alpha = torch.arange(n_alpha, dtype=torch.float64) * (2 * math.pi / n_alpha)
    gamma = torch.linspace(-max_gamma, max_gamma, n_gamma, dtype=torch.float64)
    bb, aa, cc = torch.meshgrid(beta, alpha, gamma, indexing="ij")
    return torch.stack([bb.flatten(), aa.flatten(), cc.flatten()], 1)


def s2_kernel_basis(points: Tensor, b: int):
    """Real and imaginary parts ``(P, b, 2b-1)`` of the spectra of delta kernels at ``points``."""
    points = points.to(torch.float64)
    beta, alpha = points[:, 0], points[:, 1]
    m = torch.arange(-(b - 1), b, dtype=torch.float64)
    basis = torch.zeros(points.shape[0], b, 2 * b - 1, dtype=torch.float64)
    for l in range(b):
        o = b - 1 - l
        basis[:, l, o:o + 2 * l + 1] = wigner_d(l, beta)[:, :, l]
    full = (2 * b) * basis * torch.exp(-1j * alpha[:, None] * m[None])[:, None, :]
    return full.real.contiguous(), full.imag.contiguous()


def so3_kernel_basis(points: Tensor, b: int):
    points = points.to(torch.float64)
    beta, alpha, gamma = points[:, 0], points[:, 1], points[:, 2]
    m = torch.arange(-(b - 1), b, dtype=torch.float64)
    basis = torch.zeros(points.shape[0], b, 2 * b - 1, 2 * b - 1, dtype=torch.float64)
    for l in range(b):
        o = b - 1 - l
        basis[:, l, o:o + 2 * l + 1, o:o + 2 * l + 1] = wigner_d(l, beta)
    phase = torch.exp(-1j * (alpha[:, None, None] * m[None, :, None] + gamma[:, None, None] * m[None, None, :]))
    full = basis * phase[:, None]
    return full.real.contiguous(), full.imag.contiguous()


class S2Convolution(nn.Module):
    """S2 -> SO(3) correlation with a filter of delta kernels at ``points`` (spectral product)."""

    def __init__(self, n_in: int, n_out: int, b_in: int, b_out: int, points: Tensor):
        super().__init__()
        self.n_in, self.n_out, self.b_in, self.b_out = int(n_in), int(n_out), int(b_in), int(b_out)
        self.analysis, self.synthesis = S2Transform(b_in, b_out), SO3Transform(b_out, b_out)
        re, im = s2_kernel_basis(points, b_out)
        dt = torch.get_default_dtype()
        self.register_buffer("basis_real", re.to(dt))
        self.register_buffer("basis_imag", im.to(dt))
        self.register_buffer("points", points.to(dt))
        self.kernel = nn.Parameter(torch.empty(n_in, n_out, points.shape[0]).uniform_(-1, 1))
        self.bias = nn.Parameter(torch.zeros(1, n_out, 1, 1, 1))
        self.scaling = 1.0 / math.sqrt(points.shape[0] * n_in * self.b_out ** 4 / self.b_in ** 2)

    def filter_spectrum(self) -> Tensor:
        basis = torch.complex(self.basis_real, self.basis_imag)
        return torch.einsum("iop,plm->iolm", (self.kernel * self.scaling).to(basis.dtype), basis)

    def forward(self, x: Tensor) -> Tensor:
        z = torch.einsum("bilm,ioln->bolmn", self.analysis.analyze(x), self.filter_spectrum().conj())
        return self.synthesis.synthesize(z) + self.bias


class SO3Convolution(nn.Module):
    def __init__(self, n_in: int, n_out: int, b_in: int, b_out: int, points: Tensor):
        super().__init__()
        self.n_in, self.n_out, self.b_in, self.b_out = int(n_in), int(n_out), int(b_in), int(b_out)
        self.analysis, self.synthesis = SO3Transform(b_in, b_out), SO3Transform(b_out, b_out)
        re, im = so3_kernel_basis(points, b_out)
        dt = torch.get_default_dtype()
        self.register_buffer("basis_real", re.to(dt))
        self.register_buffer("basis_imag", im.to(dt))
        self.register_buffer("points", points.to(dt))
        self.kernel = nn.Parameter(torch.empty(n_in, n_out, points.shape[0]).uniform_(-1, 1))
        self.bias = nn.Parameter(torch.zeros(1, n_out, 1, 1, 1))
        self.scaling = 1.0 / math.sqrt(points.shape[0] * n_in * self.b_out ** 3 / self.b_in ** 3)

    def filter_spectrum(self) -> Tensor:
        basis = torch.complex(self.basis_real, self.basis_imag)
        return torch.einsum("iop,plmn->iolmn", (self.kernel * self.scaling).to(basis.dtype), basis)

    def forward(self, x: Tensor) -> Tensor:
        z = torch.einsum("bilmn,iolkn->bolmk", self.analysis.analyze(x), self.filter_spectrum().conj())
        return self.synthesis.synthesize(z) + self.bias


def wigner_D(l: int, alpha, beta, gamma) -> Tensor:
    m = torch.arange(-l, l + 1, dtype=torch.float64)
    d = wigner_d(l, beta).to(torch.complex128)
    left = torch.exp(1j * torch.as_tensor(alpha, dtype=torch.float64)[..., None] * m)
    right = torch.exp(1j * torch.as_tensor(gamma, dtype=torch.float64)[..., None] * m)
    return left[..., :, None] * d * right[..., None, :]


def _rotation_blocks(b: int, alpha, beta, gamma) -> Tensor:
    out = torch.zeros(b, 2 * b - 1, 2 * b - 1, dtype=torch.complex128)
    for l in range(b):
        o = b - 1 - l
        out[l, o:o + 2 * l + 1, o:o + 2 * l + 1] = wigner_D(l, alpha, beta, gamma).conj()
    return out


def so3_rotate(x: Tensor, alpha: float, beta: float, gamma: float) -> Tensor:
    b = x.shape[-1] // 2
    tr = SO3Transform(b, b).to(x.device)
    blocks = _rotation_blocks(b, alpha, beta, gamma).to(device=x.device)
    f = tr.analyze(x)
    return tr.synthesize(torch.einsum("lmk,...lkn->...lmn", blocks.to(f.dtype), f))


def s2_rotate(x: Tensor, alpha: float, beta: float, gamma: float) -> Tensor:
    b = x.shape[-1] // 2
    tr = S2Transform(b, b).to(x.device)
    f = tr.analyze(x)
    return tr.synthesize(torch.einsum("lmk,...lk->...lm", _rotation_blocks(b, alpha, beta, gamma).to(x.device, f.dtype), f))


def euler_to_matrix(alpha, beta, gamma) -> Tensor:
    a, b, g = (float(v) for v in (alpha, beta, gamma))

    def z(t):
        return torch.tensor([[math.cos(t), -math.sin(t), 0.0], [math.sin(t), math.cos(t), 0.0], [0.0, 0.0, 1.0]],
                            dtype=torch.float64)
    y = torch.tensor([[math.cos(b), 0.0, math.sin(b)], [0.0, 1.0, 0.0], [-math.sin(b), 0.0, math.cos(b)]],
                     dtype=torch.float64)
    return z(a) @ y @ z(g)


def matrix_to_euler(R: Tensor) -> Tuple[float, float, float]:
    R = torch.as_tensor(R, dtype=torch.float64)
    beta = math.acos(max(-1.0, min(1.0, float(R[2, 2]))))
    if abs(math.sin(beta)) < 1e-9:
        sign = 1.0 if float(R[2, 2]) > 0 else -1.0
        return math.atan2(sign * float(R[1, 0]), sign * float(R[0, 0])), beta, 0.0
    return math.atan2(float(R[1, 2]), float(R[0, 2])), beta, math.atan2(float(R[2, 1]), -float(R[2, 0]))


class SphericalGrid(nn.Module):
    """Per atom and neighbour species, ``sum_j Z_i Z_j / |p - r_ij|^k`` at the ``(2b)^2`` points ``p``
    of a sphere of radius ``radius`` (optionally times a cosine cutoff of ``|r_ij|``)."""

    def __init__(self, species: Sequence[int], cutoff: float = 10.0, radius: float = 0.48, bandwidth: int = 10,
                 exponent: float = 1.0, cutoff_fn: Optional[str] = None):
        super().__init__()
        if cutoff_fn not in (None, "cosine"):
            raise ValueError(f"cutoff_fn must be None or 'cosine', got {cutoff_fn!r}")
        if bandwidth < 1 or radius <= 0:
            raise ValueError("bandwidth must be positive and radius larger than zero")
        self.species = [int(z) for z in species]
        if len(set(self.species)) != len(self.species):
            raise ValueError("species must not repeat")
        self.cutoff, self.radius, self.bandwidth, self.exponent = float(cutoff), float(radius), int(bandwidth), float(exponent)
        self.envelope = CosineCutoff(self.cutoff) if cutoff_fn == "cosine" else None
        index = torch.full((_MAX_Z,), -1, dtype=torch.long)
        for c, z in enumerate(self.species):
            index[z] = c
        self.register_buffer("species_index", index)
        self.register_buffer("directions", s2_grid_points(self.bandwidth).to(torch.get_default_dtype()))

    @property
    def n_channels(self) -> int:
        return len(self.species)

    @property
    def grid_size(self) -> int:
        return 2 * self.bandwidth

    def potential(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor) -> Tensor:
        n, nc, s = atomic_numbers.shape[0], self.n_channels, self.grid_size
        ch = self.species_index[atomic_numbers]
        if bool((ch < 0).any()):
            raise ValueError(f"atomic numbers {sorted(set(atomic_numbers[ch < 0].tolist()))} have no channel "
                             f"(species={self.species})")
        pts = (self.radius * self.directions.to(edge_vec.dtype)).reshape(-1, 3)
        src, dst = edge_index[0], edge_index[1]
        rel = -edge_vec
        q = (atomic_numbers[dst] * atomic_numbers[src]).to(edge_vec.dtype)
        if self.envelope is not None:
            q = q * self.envelope(torch.linalg.norm(rel, dim=-1))
        grid = torch.zeros(n * nc, pts.shape[0], dtype=edge_vec.dtype, device=edge_vec.device)
        row = dst * nc + ch[src]
        step = max(1, POINT_BLOCK // max(1, pts.shape[0]))
        for e0 in range(0, rel.shape[0], step):
            r = rel[e0:e0 + step]
            val = q[e0:e0 + step, None] / torch.linalg.norm(pts[None] - r[:, None], dim=-1) ** self.exponent
            grid = grid.index_add(0, row[e0:e0 + step], val)
        return grid.view(n, nc, s, s)

    def voxelize(self, atomic_numbers, edge_index, edge_vec):
        return self.potential(atomic_numbers, edge_index, edge_vec)

    def forward(self, data: AtomicGraph) -> Tensor:
        return self.potential(data.atomic_numbers, data.edge_index, data.edge_vectors())


class SphericalResBlock(nn.Module):
    def __init__(self, n_in: int, n_out: int, b_in: int, b_out: int, s2_input: bool, n_alpha: Optional[int] = None,
                 n_beta: int = 2, n_gamma: int = 2, max_beta: float = math.pi / 8,
                 normalization: Optional[str] = "batch", activation: str = "relu"):
        super().__init__()
        if normalization not in (None, "batch"):
            raise ValueError(f"normalization must be None or 'batch', got {normalization!r}")
        n_alpha = 2 * b_in if n_alpha is None else int(n_alpha)
        so3_pts = so3_near_identity_grid(max_beta, 2 * math.pi, n_alpha, n_beta, n_gamma)
        if s2_input:
            self.conv1 = S2Convolution(n_in, n_out, b_in, b_out, s2_near_identity_grid(max_beta, n_alpha, n_beta))
            self.shortcut = S2Convolution(n_in, n_out, b_in, b_out, torch.zeros(1, 2, dtype=torch.float64))
        else:
            self.conv1 = SO3Convolution(n_in, n_out, b_in, b_out, so3_pts)
            self.shortcut = (SO3Convolution(n_in, n_out, b_in, b_out, torch.zeros(1, 3, dtype=torch.float64))
                             if (n_in != n_out or b_in != b_out) else None)
        self.conv2 = SO3Convolution(n_out, n_out, b_out, b_out,
                                    so3_near_identity_grid(max_beta, 2 * math.pi, 2 * b_out, n_beta, n_gamma))
        self.norm1 = nn.BatchNorm3d(n_out) if normalization == "batch" else None
        self.norm2 = nn.BatchNorm3d(n_out) if normalization == "batch" else None
        self.act = make_activation(activation)

    def forward(self, x: Tensor) -> Tensor:
        y = self.conv1(x)
        if self.norm1 is not None:
            y = self.norm1(y)
        y = self.conv2(self.act(y))
        if self.norm2 is not None:
            y = self.norm2(y)
        return y + (x if self.shortcut is None else self.shortcut(x))


def default_schedule(n_features: int, n_blocks: int, bandwidth: int):
    feats = [max(1, round(n_features * (t + 1) / n_blocks)) for t in range(n_blocks)]
    bws = [max(2, round(bandwidth - (bandwidth - 2) * t / max(1, n_blocks - 1))) for t in range(n_blocks)]
    return feats, bws


@register_model("s2cnn")
class SphericalCNN(VoxelPotential):
    def __init__(self, species: Sequence[int] = (1, 6, 7, 8, 16), cutoff: float = 10.0, radius: float = 0.48,
                 bandwidth: int = 10, exponent: float = 1.0, features: Optional[Sequence[int]] = None,
                 bandwidths: Optional[Sequence[int]] = None, n_features: int = 160, n_blocks: int = 5,
                 n_alpha: Optional[int] = None, n_beta: int = 2, n_gamma: int = 2, max_beta: float = math.pi / 8,
                 normalization: Optional[str] = "batch", activation: str = "relu",
                 set_readout: Optional[Sequence[int]] = None, cutoff_fn: Optional[str] = None,
                 readout_activation: str = "ssp", energy_shift: float = 0.0, energy_scale: float = 1.0,
                 atomic_energies=None):
        if features is None and bandwidths is None and n_features == 160 and n_blocks == 5 and bandwidth == 10:
            features, bandwidths = [20, 40, 60, 80, 160], [10, 8, 6, 4, 2]
        if features is None or bandwidths is None:
            fd, bd = default_schedule(n_features, n_blocks, bandwidth)
            features, bandwidths = (fd if features is None else features), (bd if bandwidths is None else bandwidths)
        features, bandwidths = [int(f) for f in features], [int(b) for b in bandwidths]
        if len(features) != len(bandwidths) or not features:
            raise ValueError("features and bandwidths must have one entry per block")
        if bandwidths[0] > bandwidth or any(b1 > b0 for b0, b1 in zip(bandwidths, bandwidths[1:])):
            raise ValueError("bandwidths must not increase from block to block")
        featurizer = SphericalGrid(species, cutoff, radius, bandwidth, exponent, cutoff_fn)
        super().__init__(species, cutoff, n_features=features[-1], readout_activation=readout_activation,
                         energy_shift=energy_shift, energy_scale=energy_scale, atomic_energies=atomic_energies,
                         featurizer=featurizer)
        self.features, self.bandwidths, self.bandwidth = features, bandwidths, int(bandwidth)
        blocks, n_in, b_in = [], self.n_channels, int(bandwidth)
        for t, (n_out, b_out) in enumerate(zip(features, bandwidths)):
            blocks.append(SphericalResBlock(n_in, n_out, b_in, b_out, t == 0, n_alpha, n_beta, n_gamma, max_beta,
                                            normalization, activation))
            n_in, b_in = n_out, b_out
        self.blocks = nn.Sequential(*blocks)
        self.set_readout = None
        if set_readout is not None:
            ph, latent, ps = (int(v) for v in set_readout)
            self.set_readout = nn.ModuleDict({
                "phi": nn.Sequential(nn.Linear(features[-1], ph), make_activation(activation), nn.Linear(ph, latent),
                                     make_activation(activation)),
                "psi": nn.Sequential(nn.Linear(latent, ps), make_activation(activation), nn.Linear(ps, 1))})

    def trunk(self, grid: Tensor) -> Tensor:
        return so3_integrate(self.blocks(grid))

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        if self.set_readout is None:
            return super().forward(data)
        f = self.trunk(self.featurizer(data))
        latent = self.set_readout["phi"](f)
        pooled = latent.new_zeros(data.num_graphs, latent.shape[1]).index_add(0, data.batch, latent)
        resid = self.energy_scale * self.set_readout["psi"](pooled).squeeze(-1) + self.energy_shift * data.n_atoms.to(latent.dtype)
        node = resid[data.batch] / data.n_atoms.to(latent.dtype)[data.batch] + self.atom_ref(data.atomic_numbers).squeeze(-1)
        return {"node_energy": node, "energy": self.aggregate_energy(node, data), "node_features": f}

    @classmethod
    def from_config(cls, cfg) -> "SphericalCNN":
        e = dict(cfg.extra or {})
        return cls(species=[int(z) for z in e.get("species") or [1, 6, 7, 8, 16]], cutoff=cfg.cutoff,
                   radius=float(e.get("radius", 0.48)), bandwidth=int(e.get("bandwidth", 10)),
                   exponent=float(e.get("exponent", 1.0)),
                   features=None if e.get("features") is None else [int(f) for f in e["features"]],
                   bandwidths=None if e.get("bandwidths") is None else [int(b) for b in e["bandwidths"]],
                   n_features=cfg.n_features, n_blocks=cfg.n_interactions,
                   n_alpha=None if e.get("n_alpha") is None else int(e["n_alpha"]), n_beta=int(e.get("n_beta", 2)),
                   n_gamma=int(e.get("n_gamma", 2)), max_beta=float(e.get("max_beta", math.pi / 8)),
                   normalization=e.get("normalization", "batch"), activation=e.get("activation", "relu"),
                   set_readout=None if e.get("set_readout") is None else [int(v) for v in e["set_readout"]],
                   cutoff_fn=e.get("cutoff_fn"), readout_activation=e.get("readout_activation", "ssp"),
                   energy_shift=float(e.get("energy_shift", 0.0)), energy_scale=float(e.get("energy_scale", 1.0)),
                   atomic_energies=e.get("atomic_energies"))
