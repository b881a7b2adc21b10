"""Inverse interatomic distances ``1 / |r_a - r_b|`` over the pairs ``a > b`` (lower triangle,
row-major), with minimum-image differences in a periodic cell."""
from __future__ import annotations

from typing import Optional, Sequence

import torch
from torch import Tensor


class InverseDistances(torch.nn.Module):
    def __init__(self, n_atoms: int):
        super().__init__()
        self.n_atoms = int(n_atoms)
        a, b = torch.tril_indices(self.n_atoms, self.n_atoms, -1)
        self.register_buffer("pairs", torch.stack([a, b]), persistent=False)
        self.register_buffer("_first", a, persistent=False)
        self.register_buffer("_second", b, persistent=False)
        self.dim = int(a.numel())

    def differences(self, pos: Tensor, cell: Optional[Tensor] = None) -> Tensor:
        d = pos.index_select(1, self._first) - pos.index_select(1, self._second)
        if cell is not None:
            frac = torch.einsum("bdi,bij->bdj", d, torch.linalg.inv(cell))
            d = d - torch.einsum("bdi,bij->bdj", torch.round(frac), cell)
        return d

    def forward(self, pos: Tensor, cell: Optional[Tensor] = None) -> Tensor:
        return 1.0 / self.differences(pos, cell).norm(dim=-1)

    def pair_gradients(self, pos: Tensor, cell: Optional[Tensor] = None) -> Tensor:
        """``d x_d / d r_a`` of every pair (``-d / |d|^3``; the other atom gets the negative)."""
        d = self.differences(pos, cell)
        return -d / d.norm(dim=-1, keepdim=True) ** 3

    def permutation_index(self, perms: Sequence[Sequence[int]]) -> Tensor:
        """For every atom permutation the descriptor entry each entry moves to."""
        a, b = self.pairs.tolist()
        look = {}
        for k, (i, j) in enumerate(zip(a, b)):
            look[(i, j)] = look[(j, i)] = k
        return torch.tensor([[look[(int(p[i]), int(p[j]))] for i, j in zip(a, b)] for p in perms],
                            dtype=torch.long).reshape(len(perms), self.dim)
