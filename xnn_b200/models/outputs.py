"""Conservative forces and the stress tensor for any model.

``F = -dE/dpos`` and ``sigma = (1/V) dE/d(strain)`` with the symmetric-strain trick:
a zero ``strain (B, 3, 3)`` with ``requires_grad`` displaces positions and cells
(``src/xnn/common/models/outputs.py:96-239``). In training mode the gradient keeps its
graph (``create_graph``) so force and stress losses train the weights. Molecules of a
batch that mixes them with cells get zero stress. A model may return ``forces``
itself (direct-force models); then only the stress is taken by autograd.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..ops.modes import force_pass
from ..ops.scatter import cell_volume


class ForceStressOutput(nn.Module):
    def __init__(self, model: nn.Module, compute_forces: bool = True, compute_stress: bool = False):
        super().__init__()
        self.model = model
        self.compute_forces = compute_forces
        self.compute_stress = compute_stress
        self.cutoff = getattr(model, "cutoff", None)

    def _model_dtype(self) -> Optional[torch.dtype]:
        for t in self.model.parameters():
            if t.is_floating_point():
                return t.dtype
        for t in self.model.buffers():
            if t.is_floating_point():
                return t.dtype
        return None

    def forward(self, data: AtomicGraph, plan=None) -> dict:
        create_graph = self.training
        if data.compute_dtype is None:
            dt = self._model_dtype()
            if dt is not None and dt != data.pos.dtype:
                data.compute_dtype = dt
        strain = None
        if self.compute_stress and data.cell is not None:
            strain = torch.zeros((data.num_graphs, 3, 3), dtype=data.pos.dtype,
                                 device=data.pos.device, requires_grad=True)
            sym = 0.5 * (strain + strain.transpose(-1, -2))
            if data.num_graphs == 1:
                data.pos = data.pos + data.pos @ sym[0]
            else:
                data.pos = data.pos + torch.einsum("ni,nij->nj", data.pos,
                                                   sym.index_select(0, data.batch))
            data.cell = data.cell + torch.einsum("bki,bij->bkj", data.cell, sym)
        if self.compute_forces and not data.pos.requires_grad:
            data.pos.requires_grad_(True)
        out = self.model(data) if plan is None else self.model(data, plan)
        if "energy" not in out:
            return out
        energy = out["energy"]
        direct = "forces" in out
        inputs, need = [], []
        if self.compute_forces and not direct:
            inputs.append(data.pos)
            need.append("pos")
        if strain is not None:
            inputs.append(strain)
            need.append("strain")
        g = {k: None for k in need}
        if inputs and energy.requires_grad:
            # only position / strain derivatives are asked for: the fused ops skip the rest
            with force_pass():
                grads = torch.autograd.grad([energy], inputs, grad_outputs=[torch.ones_like(energy)],
                                            create_graph=create_graph, retain_graph=create_graph,
                                            allow_unused=True)
            g = dict(zip(need, grads))
        if self.compute_forces and not direct:
            out["forces"] = -g["pos"] if g.get("pos") is not None else torch.zeros_like(data.pos)
        if strain is not None:
            sg = g.get("strain")
            out["stress"] = _stress(sg, data) if sg is not None else torch.zeros_like(strain)
        return out


def _stress(strain_gradient: Tensor, data: AtomicGraph) -> Tensor:
    volume = cell_volume(data.cell)
    periodic = volume > 1e-8
    if data.pbc is not None:
        periodic = periodic & data.pbc.any(-1).to(periodic.device)
    safe = torch.where(periodic, volume, torch.ones_like(volume))
    return torch.where(periodic[:, None, None], strain_gradient / safe[:, None, None].to(strain_gradient.dtype),
                       torch.zeros_like(strain_gradient))
