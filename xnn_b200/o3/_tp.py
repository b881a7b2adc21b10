"""Weighted tensor products of irreps with e3nn's instruction format and normalisation.

An instruction ``(i_in1, i_in2, i_out, mode, has_weight[, path_weight])`` couples one
block of each input into one output block through the Clebsch-Gordan tensor
``wigner_3j(l1, l2, l_out)``. The connection modes and the ``"component"`` /
``"element"`` normalisation (each path scaled by ``sqrt(dim_out / fan_in)``, the fan-in
counting every path into the same output block) reproduce e3nn's ``o3.TensorProduct``,
whose flat per-instruction weight layout the reference's MACE and NequIP
convolutions (``src/xnn/gnn/fast/conv.py:22-50``) and self-connections
(``src/xnn/gnn/fast/linear.py:160-190``) store.
"""
from __future__ import annotations

import math
from typing import List, NamedTuple, Optional

import torch
from torch import Tensor, nn

from ._irreps import Irreps
from ._wigner import wigner_3j


class Instruction(NamedTuple):
    i_in1: int
    i_in2: int
    i_out: int
    connection_mode: str
    has_weight: bool
    path_weight: float
    path_shape: tuple


def _num_elements(mode: str, mul1: int, mul2: int) -> int:
    return {"uvw": mul1 * mul2, "uvu": mul2, "uvv": mul1, "uuw": mul1, "uuu": 1,
            "uvuv": 1}[mode]


def _path_shape(mode: str, mul1: int, mul2: int, mul_out: int) -> tuple:
    return {"uvw": (mul1, mul2, mul_out), "uvu": (mul1, mul2), "uvv": (mul1, mul2),
            "uuw": (mul1, mul_out), "uuu": (mul1,), "uvuv": (mul1, mul2)}[mode]


class TensorProduct(nn.Module):
    """Tensor product ``irreps_in1 x irreps_in2 -> irreps_out`` along explicit instructions."""

    def __init__(self, irreps_in1, irreps_in2, irreps_out, instructions, in1_var=None,
                 in2_var=None, out_var=None, irrep_normalization: str = "component",
                 path_normalization: str = "element", internal_weights: Optional[bool] = None,
                 shared_weights: Optional[bool] = None):
        super().__init__()
        self.irreps_in1 = Irreps(irreps_in1)
        self.irreps_in2 = Irreps(irreps_in2)
        self.irreps_out = Irreps(irreps_out)
        in1_var = in1_var or [1.0] * len(self.irreps_in1)
        in2_var = in2_var or [1.0] * len(self.irreps_in2)
        out_var = out_var or [1.0] * len(self.irreps_out)
        raw = [tuple(ins) + ((1.0,) if len(ins) == 5 else ()) for ins in instructions]

        def norm(ins) -> float:
            i1, i2, io, mode, _w, pw = ins
            m1, m2, mo = self.irreps_in1[i1], self.irreps_in2[i2], self.irreps_out[io]
            if irrep_normalization == "component":
                alpha = mo.ir.dim
            elif irrep_normalization == "norm":
                alpha = m1.ir.dim * m2.ir.dim
            else:
                alpha = 1.0
            if path_normalization == "element":
                x = sum(in1_var[j[0]] * in2_var[j[1]]
                        * _num_elements(j[3], self.irreps_in1[j[0]].mul, self.irreps_in2[j[1]].mul)
                        for j in raw if j[2] == io)
            elif path_normalization == "path":
                x = in1_var[i1] * in2_var[i2] * _num_elements(mode, m1.mul, m2.mul)
                x *= len([j for j in raw if j[2] == io])
            else:
                x = 1.0
            if x > 0:
                alpha /= x
            alpha *= out_var[io]
            alpha *= pw
            return math.sqrt(alpha)

        self.instructions: List[Instruction] = []
        for ins in raw:
            i1, i2, io, mode, has_w, _ = ins
            m1, m2, mo = self.irreps_in1[i1], self.irreps_in2[i2], self.irreps_out[io]
            if mo.ir not in list(m1.ir * m2.ir):
                raise ValueError(f"instruction {ins} has no coupling path")
            self.instructions.append(Instruction(i1, i2, io, mode, bool(has_w), norm(ins),
                                                 _path_shape(mode, m1.mul, m2.mul, mo.mul)))
        if shared_weights is False and internal_weights is None:
            internal_weights = False
        if shared_weights is None:
            shared_weights = True
        if internal_weights is None:
            internal_weights = shared_weights and any(i.has_weight for i in self.instructions)
        self.internal_weights = internal_weights
        self.shared_weights = shared_weights
        self.weight_numel = sum(math.prod(i.path_shape) for i in self.instructions if i.has_weight)
        if internal_weights and self.weight_numel > 0:
            self.weight = nn.Parameter(torch.randn(self.weight_numel))
        else:
            self.register_buffer("weight", torch.Tensor())
        mask = [torch.ones(m.dim) if any(i.i_out == o and i.path_weight != 0 for i in self.instructions)
                else torch.zeros(m.dim) for o, m in enumerate(self.irreps_out)]
        self.register_buffer("output_mask", torch.cat(mask) if mask else torch.ones(0))
        # coupling tensors kept out of the state dict, built per (dtype, device) on use
        self.__dict__["_cg_cache"] = {}

    def _cg(self, l1: int, l2: int, lo: int, like: Tensor) -> Tensor:
        key = (l1, l2, lo, like.dtype, like.device)
        cache = self.__dict__["_cg_cache"]
        if key not in cache:
            cache[key] = wigner_3j(l1, l2, lo, dtype=like.dtype, device=like.device)
        return cache[key]

    def weight_views(self, weight: Optional[Tensor] = None, yield_instruction: bool = False):
        """The weights of each weighted instruction as views of shape ``(..., *path_shape)``
        (the module's own weights by default)."""
        if weight is None:
            weight = self.weight
        batch = weight.shape[:-1]
        at = 0
        for ins in self.instructions:
            if not ins.has_weight:
                continue
            n = math.prod(ins.path_shape)
            view = weight.narrow(-1, at, n).view(batch + tuple(ins.path_shape))
            at += n
            yield (ins, view) if yield_instruction else view

    def __repr__(self) -> str:
        return (f"TensorProduct({self.irreps_in1} x {self.irreps_in2} -> {self.irreps_out} | "
                f"{len(self.instructions)} paths | {self.weight_numel} weights)")

    def forward(self, x1: Tensor, x2: Tensor, weight: Optional[Tensor] = None) -> Tensor:
        if weight is None:
            if self.weight_numel > 0 and not self.internal_weights:
                raise RuntimeError("weights must be given when internal_weights=False")
            weight = self.weight
        lead = torch.broadcast_shapes(x1.shape[:-1], x2.shape[:-1])
        x1 = x1.expand(*lead, x1.shape[-1]).reshape(-1, self.irreps_in1.dim)
        x2 = x2.expand(*lead, x2.shape[-1]).reshape(-1, self.irreps_in2.dim)
        n = x1.shape[0]
        if self.weight_numel > 0:
            per_sample = weight.dim() > 1
            w_all = weight.reshape(n, -1) if per_sample else weight
        s1, s2 = self.irreps_in1.slices(), self.irreps_in2.slices()
        outs: List[Optional[Tensor]] = [None] * len(self.irreps_out)
        off = 0
        for ins in self.instructions:
            m1, m2, mo = (self.irreps_in1[ins.i_in1], self.irreps_in2[ins.i_in2],
                          self.irreps_out[ins.i_out])
            a = x1[:, s1[ins.i_in1]].reshape(n, m1.mul, m1.ir.dim)
            b = x2[:, s2[ins.i_in2]].reshape(n, m2.mul, m2.ir.dim)
            cg = self._cg(m1.ir.l, m2.ir.l, mo.ir.l, a)
            mode = ins.connection_mode
            if ins.has_weight:
                numel = math.prod(ins.path_shape)
                w = (w_all[:, off:off + numel] if per_sample else w_all[off:off + numel])
                w = w.reshape(((n,) if per_sample else ()) + ins.path_shape)
                off += numel
            pre = "n" if (ins.has_weight and per_sample) else ""
            if mode == "uvw":
                y = (torch.einsum(f"nui,nvj,ijk,{pre}uvw->nwk", a, b, cg, w) if ins.has_weight
                     else None)
                if y is None:
                    raise ValueError("uvw paths need weights")
            elif mode == "uvu":
                if ins.has_weight:
                    y = torch.einsum(f"nui,nvj,ijk,{pre}uv->nuk", a, b, cg, w)
                else:
                    y = torch.einsum("nui,nvj,ijk->nuk", a, b, cg)
            elif mode == "uvv":
                if ins.has_weight:
                    y = torch.einsum(f"nui,nvj,ijk,{pre}uv->nvk", a, b, cg, w)
                else:
                    y = torch.einsum("nui,nvj,ijk->nvk", a, b, cg)
            elif mode == "uuw":
                if ins.has_weight:
                    y = torch.einsum(f"nui,nuj,ijk,{pre}uw->nwk", a, b, cg, w)
                else:
                    y = torch.einsum("nui,nuj,ijk->nk", a, b, cg)[:, None].expand(n, mo.mul, -1)
            elif mode == "uuu":
                if ins.has_weight:
                    y = torch.einsum(f"nui,nuj,ijk,{pre}u->nuk", a, b, cg, w)
                else:
                    y = torch.einsum("nui,nuj,ijk->nuk", a, b, cg)
            elif mode == "uvuv":
                if ins.has_weight:
                    y = torch.einsum(f"nui,nvj,ijk,{pre}uv->nuvk", a, b, cg, w)
                else:
                    y = torch.einsum("nui,nvj,ijk->nuvk", a, b, cg)
                y = y.reshape(n, -1, mo.ir.dim)
            else:
                raise ValueError(f"unknown connection mode {mode!r}")
            y = y * ins.path_weight
            outs[ins.i_out] = y if outs[ins.i_out] is None else outs[ins.i_out] + y
        pieces = []
        for o, m in enumerate(self.irreps_out):
            blk = outs[o]
            if blk is None:
                blk = x1.new_zeros(n, m.mul, m.ir.dim)
            pieces.append(blk.reshape(n, m.dim))
        out = torch.cat(pieces, -1) if len(pieces) > 1 else pieces[0]
        return out.reshape(*lead, self.irreps_out.dim)


class FullyConnectedTensorProduct(TensorProduct):
    """Every ``uvw`` path of ``irreps_in1 x irreps_in2`` that lands in ``irreps_out``."""

    def __init__(self, irreps_in1, irreps_in2, irreps_out, **kwargs):
        i1, i2, io = Irreps(irreps_in1), Irreps(irreps_in2), Irreps(irreps_out)
        ins = [(a, b, c, "uvw", True, 1.0)
               for a, m1 in enumerate(i1) for b, m2 in enumerate(i2) for c, mo in enumerate(io)
               if mo.ir in list(m1.ir * m2.ir)]
        super().__init__(i1, i2, io, ins, **kwargs)
