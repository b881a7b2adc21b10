"""Neighbour lists with periodic images.

Semantics follow the reference's ``build_neighbor_list``
(``src/xnn/common/data/neighborlist.py:411-506``): edges ``[src, dst]`` with ``dst``
the receiver, pairs strictly inside the cutoff, self pairs only in non-zero images,
positions wrapped into the cell along periodic axes with the integer offsets folded
back into ``cell_shifts`` so unwrapped trajectories work, and the edge vector
``pos[dst] - pos[src] + shift @ cell`` equal to the selecting displacement.

Three engines produce identical edge sets: the native cell list of
``xnn_b200._C`` (CUDA on a GPU, C++/OpenMP on the CPU; count, prefix sum, write, so
the edges come out grouped by receiver in a deterministic order), and a blocked
brute-force PyTorch fallback used when the extension is absent on the CPU. The
result is always sorted by receiver, then sender, then shift.
"""
from __future__ import annotations

import itertools
import math
from typing import Optional, Tuple

import torch
from torch import Tensor


def _n_repeats(cell: Tensor, cutoff: float, pbc: Tensor) -> Tuple[int, int, int]:
    """Images per axis needed to see every neighbour within ``cutoff`` (plane distances)."""
    c = cell.to(torch.float64)
    vol = torch.linalg.det(c).abs()
    reps = []
    for a in range(3):
        b, d = c[(a + 1) % 3], c[(a + 2) % 3]
        height = vol / torch.linalg.cross(b, d).norm()
        reps.append(int(math.ceil(cutoff / float(height))) if bool(pbc[a]) else 0)
    return tuple(reps)  # type: ignore[return-value]


def _wrap(pos: Tensor, cell: Tensor, pbc: Tensor) -> Tuple[Tensor, Tensor]:
    frac = pos.to(torch.float64) @ torch.linalg.inv(cell.to(torch.float64))
    off = torch.floor(frac).to(torch.long)
    off[:, ~pbc.to(torch.bool).to(off.device)] = 0
    wrapped = pos - off.to(pos.dtype) @ cell.to(pos.dtype)
    return wrapped, off


def _sort_edges(edge_index: Tensor, shifts: Tensor, n: int) -> Tuple[Tensor, Tensor]:
    if edge_index.shape[1] == 0:
        return edge_index, shifts
    sk = ((shifts[:, 0] + 64) * 129 + (shifts[:, 1] + 64)) * 129 + (shifts[:, 2] + 64)
    key = (edge_index[1] * n + edge_index[0]) * (129 ** 3) + sk
    order = torch.argsort(key)
    return edge_index[:, order], shifts[order]


def _brute_force(pos: Tensor, cutoff: float, cell: Optional[Tensor], pbc: Optional[Tensor],
                 self_interaction: bool, block: int = 2048) -> Tuple[Tensor, Tensor]:
    device, dtype = pos.device, pos.dtype
    n = pos.shape[0]
    offsets = None
    if cell is None or pbc is None or not bool(pbc.any()):
        shift_idx = torch.zeros((1, 3), device=device, dtype=torch.long)
    else:
        pos, offsets = _wrap(pos, cell, pbc)
        reps = _n_repeats(cell, cutoff, pbc)
        combos = list(itertools.product(*[range(-r, r + 1) for r in reps]))
        shift_idx = torch.tensor(combos, device=device, dtype=torch.long)
    shifts = shift_idx.to(dtype) @ cell.to(dtype) if cell is not None and offsets is not None \
        else torch.zeros((1, 3), device=device, dtype=dtype)
    srcs, dsts, sh = [], [], []
    zero_shift = (shift_idx == 0).all(dim=1)
    for i0 in range(0, n, block):
        i1 = min(n, i0 + block)
        # displacement from receiver i to sender j in image s: pos[j] - pos[i] + shift
        rij = pos[None, None, :, :] - pos[None, i0:i1, None, :] + shifts[:, None, None, :]
        within = (rij * rij).sum(-1) < cutoff * cutoff
        if not self_interaction:
            eye = torch.zeros(i1 - i0, n, dtype=torch.bool, device=device)
            eye[torch.arange(i1 - i0, device=device), torch.arange(i0, i1, device=device)] = True
            within &= ~(eye[None] & zero_shift[:, None, None])
        s_idx, i_idx, j_idx = torch.nonzero(within, as_tuple=True)
        srcs.append(j_idx)
        dsts.append(i_idx + i0)
        sh.append(-shift_idx[s_idx])
    src = torch.cat(srcs)
    dst = torch.cat(dsts)
    cell_shifts = torch.cat(sh)
    if offsets is not None:
        cell_shifts = cell_shifts + offsets[src] - offsets[dst]
    return torch.stack([src, dst]), cell_shifts


def build_neighbor_list(pos: Tensor, cutoff: float, cell: Optional[Tensor] = None,
                        pbc: Optional[Tensor] = None, self_interaction: bool = False,
                        engine: str = "auto", receivers: Optional[Tuple[int, int]] = None) -> Tuple[Tensor, Tensor]:
    """``(edge_index (2, E), cell_shifts (E, 3))`` of one structure (see module notes).

    Parameters
    ----------
    engine : {"auto", "native", "torch"}
        ``"auto"`` takes the native cell list when the extension is loaded.
    receivers : (int, int), optional
        Only edges into atoms ``r0 <= i < r1`` (every atom stays a candidate sender): one
        process's share of a list split over processes.
    """
    if cell is not None and cell.dim() == 3:
        cell = cell[0]
    if pbc is not None and pbc.dim() == 2:
        pbc = pbc[0]
    if pbc is not None:
        pbc = pbc.to(torch.bool).cpu()
    periodic = cell is not None and pbc is not None and bool(pbc.any())
    if engine in ("auto", "native"):
        from .. import _ext
        if _ext.available() or engine == "native":
            return _native(pos, cutoff, cell if periodic else None, pbc if periodic else None,
                           self_interaction, receivers)
    ei, sh = _brute_force(pos, cutoff, cell if periodic else None, pbc if periodic else None,
                          self_interaction)
    ei, sh = _sort_edges(ei, sh, pos.shape[0])
    if receivers is not None:
        keep = (ei[1] >= receivers[0]) & (ei[1] < receivers[1])
        ei, sh = ei[:, keep], sh[keep]
    return ei, sh


def _native(pos: Tensor, cutoff: float, cell: Optional[Tensor], pbc: Optional[Tensor],
            self_interaction: bool, receivers: Optional[Tuple[int, int]] = None) -> Tuple[Tensor, Tensor]:
    from .. import _ext
    C = _ext.ops()
    p64 = pos.detach().to(torch.float64).contiguous()
    offsets = None
    if cell is not None:
        p64, offsets = _wrap(p64, cell.to(p64.device), pbc)
        reps = torch.tensor(_n_repeats(cell, cutoff, pbc), dtype=torch.long)
        cell64 = cell.detach().to(torch.float64).to(p64.device).contiguous()
        pbc_t = pbc.to(torch.long)
    else:
        reps = torch.zeros(3, dtype=torch.long)
        cell64 = torch.zeros(3, 3, dtype=torch.float64, device=p64.device)
        pbc_t = torch.zeros(3, dtype=torch.long)
    r0, r1 = (0, -1) if receivers is None else (int(receivers[0]), int(receivers[1]))
    src, dst, shifts = C.neighbor_list(p64, cell64, [int(r) for r in reps], [int(b) for b in pbc_t],
                                       float(cutoff), bool(self_interaction), r0, r1)
    if offsets is not None:
        shifts = shifts + offsets[src] - offsets[dst]
    return torch.stack([src, dst]), shifts


def unique_pairs(edge_index: Tensor, cell_shifts: Tensor) -> Tuple[Tensor, Tensor]:
    """Half list ``i < k`` (or ``i == k`` with a positive image) of a full list, sorted by ``i``."""
    src, dst = edge_index
    s = cell_shifts
    first_nonzero = torch.where(s[:, 0] != 0, s[:, 0], torch.where(s[:, 1] != 0, s[:, 1], s[:, 2]))
    keep = (dst < src) | ((dst == src) & (first_nonzero > 0))
    ei = torch.stack([dst[keep], src[keep]])
    sh = -s[keep]
    order = torch.argsort(ei[0] * (int(ei.max()) + 1 if ei.numel() else 1) + ei[1], stable=True)
    return ei[:, order], sh[order]


def nearest_edges(edge_index: Tensor, lengths: Tensor, k: int, n_nodes: int) -> Tensor:
    """Mask keeping the ``k`` shortest incoming edges of every receiver (CGCNN's graph)."""
    dst = edge_index[1]
    order = torch.argsort(lengths, stable=True)
    order = order[torch.argsort(dst[order], stable=True)]
    counts = torch.bincount(dst, minlength=n_nodes)
    starts = torch.cumsum(counts, 0) - counts
    rank = torch.empty_like(order)
    rank[order] = torch.arange(order.numel(), device=order.device) - starts[dst[order]]
    return rank < k
