"""Geometry of the bonded and pair terms of the classical force fields on batched conformers:
minimum-image displacements (integer image shifts found without gradient, so forces and the cell
derivative flow through ``pos[b] - pos[a] + shift @ cell``), dihedral cosines/sines from plane
normals (no ``arccos``, whose derivative is singular at planar geometries), and the neighbour
list's pairs once each with a bound topology's exclusions removed.

Conventions follow the reference (``src/xnn/ffnn/models/geometry.py:41-389``): ``phi = 0`` at
cis, the IUPAC sign of ``sin phi``, own images at half weight, a 1e-12 regulariser under square
roots.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

TINY = 1.0e-12
ORTHOGONAL_TOL = 1.0e-10


def geometric_mean(x: Tensor, y: Tensor) -> Tensor:
    """``sqrt(x y)``, exactly zero with zero gradient where the product vanishes."""
    prod = x * y
    return torch.where(prod > 0.0, torch.sqrt(torch.clamp(prod, min=TINY)), torch.zeros_like(prod))


@torch.no_grad()
def image_shifts(vec: Tensor, lattice: Tensor, pbc: Optional[Tensor]) -> Tensor:
    """Integer shifts ``(M, 3)`` minimising ``|vec + shift @ lattice|`` for one lattice ``(3, 3)``
    whose non-periodic rows are zero: the rounded fractional image, then the best of its 27
    neighbours for a skewed lattice."""
    flags = None if pbc is None else pbc.to(vec.dtype)
    inv = torch.linalg.inv_ex(lattice)[0] if pbc is None or bool(pbc.all()) else torch.linalg.pinv(lattice)
    shift = -torch.round(vec @ inv)
    if flags is not None:
        shift = shift * flags
    gram = lattice @ lattice.T
    off = gram - torch.diag(torch.diagonal(gram))
    # inside a CUDA-graph capture the 27-image search always runs (no host read of the skew test)
    if _capturing(vec) or bool((off.abs() > ORTHOGONAL_TOL * gram.abs().amax()).any()):
        one = torch.arange(-1, 2, device=vec.device)
        offs = torch.cartesian_prod(one, one, one).to(vec.dtype)
        if flags is not None:
            offs = offs * flags
        cand = vec[:, None, :] + (shift[:, None, :] + offs[None]) @ lattice
        shift = shift + offs[(cand * cand).sum(-1).argmin(1)]
    return shift


def pair_shifts(data, a: Tensor, b: Tensor) -> Optional[Tensor]:
    """Image shifts of ``pos[b] - pos[a]`` (``None`` without a cell)."""
    if data.cell is None or a.shape[0] == 0:
        return None
    vec = (data.pos[b] - data.pos[a]).detach()
    pbc = data.pbc if data.pbc is not None else torch.ones_like(data.cell[:, 0, 0], dtype=torch.bool)[:, None].expand(-1, 3)
    lattice = data.cell.detach().to(vec.dtype) * pbc.to(vec.dtype)[..., None]
    if lattice.shape[0] == 1:
        return image_shifts(vec, lattice[0], pbc[0])
    out = torch.zeros_like(vec)
    g = data.batch[a]
    for s in torch.unique(g).tolist():
        m = g == s
        out[m] = image_shifts(vec[m], lattice[s], pbc[s])
    return out


def pair_vectors(data, a: Tensor, b: Tensor, shift: Optional[Tensor] = None) -> Tensor:
    """Minimum-image ``pos[b] - pos[a]`` in the model dtype."""
    vec = data.pos.index_select(0, b) - data.pos.index_select(0, a)
    if data.cell is None or vec.shape[0] == 0:
        return vec.to(data.model_dtype)
    if shift is None:
        shift = pair_shifts(data, a, b)
    cell = data.cell.to(vec.dtype)
    if cell.shape[0] == 1:
        return (vec + (shift.to(vec.dtype)[:, :, None] * cell[0]).sum(1)).to(data.model_dtype)
    cells = cell.index_select(0, data.batch.index_select(0, a))
    return (vec + (shift.to(vec.dtype)[:, :, None] * cells).sum(1)).to(data.model_dtype)


def bond_vectors(data, idx: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
    """The three bond vectors ``b1 = x1 - x0``, ``b2 = x2 - x1``, ``b3 = x3 - x2`` of ``(4, M)``."""
    return tuple(pair_vectors(data, idx[j], idx[j + 1]) for j in range(3))


def dihedral_cos(data, idx: Tensor) -> Tensor:
    b1, b2, b3 = bond_vectors(data, idx)
    n1, n2 = torch.cross(b1, b2, dim=1), torch.cross(b2, b3, dim=1)
    return (n1 * n2).sum(1) / torch.sqrt((n1 * n1).sum(1) * (n2 * n2).sum(1) + TINY)


def dihedral_cos_sin(data, idx: Tensor) -> Tuple[Tensor, Tensor]:
    """``(cos phi, sin phi)`` with the IUPAC sign."""
    b1, b2, b3 = bond_vectors(data, idx)
    n1, n2 = torch.cross(b1, b2, dim=1), torch.cross(b2, b3, dim=1)
    norm = torch.sqrt((n1 * n1).sum(1) * (n2 * n2).sum(1) + TINY)
    b2n = torch.sqrt((b2 * b2).sum(1) + TINY)
    return (n1 * n2).sum(1) / norm, -(torch.cross(n1, n2, dim=1) * b2).sum(1) / (norm * b2n)


def angle_theta(data, idx: Tensor) -> Tensor:
    """Angle at ``idx[1]`` of ``(3, M)`` triples, clamped away from 0 and pi for a finite gradient."""
    u, v = pair_vectors(data, idx[1], idx[0]), pair_vectors(data, idx[1], idx[2])
    c = (u * v).sum(1) / torch.sqrt((u * u).sum(1) * (v * v).sum(1) + TINY)
    bound = min(0.9999999999, 1.0 - 4.0 * torch.finfo(c.dtype).eps)
    return torch.arccos(torch.clamp(c, -bound, bound))


def batch_index(idx: Tensor, n: int, b: int) -> Tensor:
    """``(k, M)`` atom indices of one structure repeated over ``b`` structures of ``n`` atoms."""
    starts = torch.arange(b, device=idx.device) * n
    return (idx.unsqueeze(1) + starts.view(1, b, 1)).reshape(idx.shape[0], -1)


def excluded(i: Tensor, k: Tensor, excl_index: Tensor, n: int, b: int, cache: dict) -> Tensor:
    """Whether each pair of the batch is one of the topology's excluded pairs (either order)."""
    if excl_index.shape[1] == 0:
        return torch.zeros(i.shape, dtype=torch.bool, device=i.device)
    N = n * b
    ck = (b, N, str(excl_index.device))
    if ck not in cache:
        ex = batch_index(excl_index, n, b)
        cache[ck] = torch.sort(torch.minimum(ex[0], ex[1]) * N + torch.maximum(ex[0], ex[1])).values
    keys = cache[ck]
    key = torch.minimum(i, k) * N + torch.maximum(i, k)
    at = torch.searchsorted(keys, key).clamp_(max=keys.shape[0] - 1)
    return keys.index_select(0, at) == key


def _capturing(t: Tensor) -> bool:
    return t.is_cuda and torch.cuda.is_current_stream_capturing()


def half_edges(data, excl_index: Tensor, n: int, cache: dict):
    """The neighbour list's pairs once each (``src <= dst``): ``src, dst``, the vectors, squared
    lengths, weights (half for an atom's own image) and whether each pair is not excluded. Inside
    a CUDA-graph capture every directed edge is kept at weight one half instead (the same sum with
    shapes that do not depend on the data)."""
    src, dst = data.edge_index[0], data.edge_index[1]
    if _capturing(src):
        vec = pair_vectors(data, src, dst, None if data.cell is None else data.cell_shifts)
        r2 = (vec * vec).sum(1)
        half = torch.full_like(r2, 0.5)
        return src, dst, vec, r2, half, ~excluded(src, dst, excl_index, n, data.num_graphs, cache)
    once = (src <= dst).nonzero()[:, 0]
    src, dst = src[once], dst[once]
    vec = pair_vectors(data, src, dst, None if data.cell is None else data.cell_shifts[once])
    r2 = (vec * vec).sum(1)
    half = torch.where(src == dst, 0.5, 1.0).to(r2.dtype)
    return src, dst, vec, r2, half, ~excluded(src, dst, excl_index, n, data.num_graphs, cache)


def quintic_switch(r: Tensor, cutoff: float, width: float) -> Tensor:
    """1 below ``cutoff - width``, ``1 - x^3 (10 - 15 x + 6 x^2)`` across the last ``width``, 0 from
    the cutoff on (pairs of a skin list beyond the cutoff count nothing)."""
    inside = (r < cutoff).to(r.dtype)
    if width <= 0.0:
        return inside
    x = torch.clamp((r - (cutoff - width)) / width, 0.0, 1.0)
    return (1.0 - x ** 3 * (10.0 - 15.0 * x + 6.0 * x * x)) * inside
