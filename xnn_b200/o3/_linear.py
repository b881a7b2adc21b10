"""Equivariant linear map between irreps, with e3nn's parameter layout.

``Linear(irreps_in, irreps_out)`` mixes the multiplicities of every pair of equal
irreps. One flat ``weight`` parameter holds the ``(mul_in, mul_out)`` matrix of
each path in path order; a path into output block ``o`` is scaled by
``1 / sqrt(sum of mul_in over the paths into o)``. The state-dict entries
(``weight``, ``bias``, ``output_mask``) are those of e3nn's ``o3.Linear``, which
the reference's MACE/NequIP checkpoints store (``src/xnn/gnn/fast/linear.py:106-121``).
"""
from __future__ import annotations

import math
from typing import List, NamedTuple, Optional

import torch
from torch import Tensor, nn

from ._irreps import Irreps


class LinearPath(NamedTuple):
    i_in: int
    i_out: int
    path_shape: tuple
    path_weight: float


class Linear(nn.Module):
    """Equivariant linear map ``irreps_in -> irreps_out`` (see module notes)."""

    def __init__(self, irreps_in, irreps_out, *, internal_weights: Optional[bool] = None,
                 shared_weights: Optional[bool] = None, instructions=None, biases=False,
                 path_normalization: str = "element"):
        super().__init__()
        self.irreps_in = Irreps(irreps_in)
        self.irreps_out = Irreps(irreps_out)
        if instructions is None:
            instructions = [(i, o) for i, a in enumerate(self.irreps_in)
                            for o, b in enumerate(self.irreps_out) if a.ir == b.ir]
        if isinstance(biases, bool):
            biases = [biases and b.ir.is_scalar() for b in self.irreps_out]

        def fan(i_out: int, i_in: int) -> int:
            if path_normalization == "element":
                x = sum(self.irreps_in[ii].mul for ii, oo in instructions if oo == i_out)
            else:
                x = self.irreps_in[i_in].mul
            return x if x > 0 else 1

        self.instructions: List[LinearPath] = [
            LinearPath(i, o, (self.irreps_in[i].mul, self.irreps_out[o].mul), fan(o, i) ** -0.5)
            for i, o in instructions
        ]
        self.bias_outputs = [o for o, b in enumerate(biases) if b]
        if shared_weights is False and internal_weights is None:
            internal_weights = False
        if shared_weights is None:
            shared_weights = True
        if internal_weights is None:
            internal_weights = True
        self.internal_weights = internal_weights
        self.shared_weights = shared_weights
        self.weight_numel = sum(math.prod(p.path_shape) for p in self.instructions)
        self.bias_numel = sum(self.irreps_out[o].dim for o in self.bias_outputs)
        if internal_weights and self.weight_numel > 0:
            self.weight = nn.Parameter(torch.randn(self.weight_numel))
        else:
            self.register_buffer("weight", torch.Tensor())
        if internal_weights and self.bias_numel > 0:
            self.bias = nn.Parameter(torch.zeros(self.bias_numel))
        else:
            self.register_buffer("bias", torch.Tensor())
        mask = [torch.ones(m.dim) if any(p.i_out == o for p in self.instructions)
                else torch.zeros(m.dim) for o, m in enumerate(self.irreps_out)]
        self.register_buffer("output_mask", torch.cat(mask) if mask else torch.ones(0))

    def __repr__(self) -> str:
        return f"Linear({self.irreps_in} -> {self.irreps_out} | {self.weight_numel} weights)"

    def path_matrices(self, weight: Optional[Tensor] = None) -> List[Tensor]:
        """The scaled ``(mul_in, mul_out)`` matrix of every path (shared weights only)."""
        w = self.weight if weight is None else weight
        out, off = [], 0
        for p in self.instructions:
            n = p.path_shape[0] * p.path_shape[1]
            out.append(w[off:off + n].view(p.path_shape) * p.path_weight)
            off += n
        return out

    def forward(self, x: Tensor, weight: Optional[Tensor] = None, bias: Optional[Tensor] = None) -> Tensor:
        if weight is None:
            weight = self.weight
        if bias is None:
            bias = self.bias
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.irreps_in.dim)
        n = x2.shape[0]
        in_sl = self.irreps_in.slices()
        outs: List[Optional[Tensor]] = [None] * len(self.irreps_out)
        off = 0
        for p in self.instructions:
            mi, mo = p.path_shape
            d = self.irreps_in[p.i_in].ir.dim
            blk = x2[:, in_sl[p.i_in]].reshape(n, mi, d)
            if weight.dim() == 1:
                w = weight[off:off + mi * mo].view(mi, mo)
                y = torch.einsum("nud,uw->nwd", blk, w) if d > 1 else (blk[..., 0] @ w)[..., None]
            else:  # per-sample weights
                w = weight.reshape(n, -1)[:, off:off + mi * mo].view(n, mi, mo)
                y = torch.einsum("nud,nuw->nwd", blk, w)
            y = y * p.path_weight
            outs[p.i_out] = y if outs[p.i_out] is None else outs[p.i_out] + y
            off += mi * mo
        pieces = []
        boff = 0
        for o, m in enumerate(self.irreps_out):
            blk = outs[o]
            if blk is None:
                blk = x2.new_zeros(n, m.mul, m.ir.dim)
            if o in self.bias_outputs:
                blk = blk + bias[boff:boff + m.dim].view(1, m.mul, 1)
                boff += m.dim
            pieces.append(blk.reshape(n, m.dim))
        out = torch.cat(pieces, -1) if len(pieces) > 1 else (pieces[0] if pieces else x2.new_zeros(n, 0))
        return out.reshape(*lead, self.irreps_out.dim)
