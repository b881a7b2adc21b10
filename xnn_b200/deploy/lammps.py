"""LAMMPS / TorchScript export.

The archive contract follows the reference's ``src/xnn/common/deploy/lammps.py:23-210`` so the same
pair style drives either build: a TorchScript module whose
``forward(pos, edge_index, cell_shifts, atomic_numbers, cell)`` returns ``{"total_energy" (1,),
"node_energy" (N,), "forces" (N, 3)}`` from neighbour data the host supplies, with the cutoff and
metadata stored as extra files (strings).

How it is built here: the model's energy core ``node_energy(atomic_numbers, edge_index,
edge_vec)`` runs with the fused CUDA kernels switched off and is *traced* (its operations are
plain tensor operations, so the trace is shape-generic), and a small *scripted* wrapper forms
the edge vectors and takes the forces by ``torch.autograd.grad`` around the traced core.
"""
from __future__ import annotations

import json
from typing import Dict, Optional

import torch
from torch import Tensor, nn


class _EnergyCore(nn.Module):
    def __init__(self, model: nn.Module):
        super().__init__()
        self.model = model

    def forward(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor) -> Tensor:
        return self.model.node_energy(atomic_numbers, edge_index, edge_vec)


class LAMMPSWrapper(nn.Module):
    """Energy, per-atom energies and forces from host-built neighbour data (scriptable)."""

    def __init__(self, core: nn.Module, cutoff: float, core_cutoff: float):
        super().__init__()
        self.core = core
        self.cutoff = float(cutoff)
        self.core_cutoff = float(core_cutoff)

    def forward(self, pos: Tensor, edge_index: Tensor, cell_shifts: Tensor, atomic_numbers: Tensor,
                cell: Tensor) -> Dict[str, Tensor]:
        pos = pos.detach().requires_grad_(True)
        vec = pos[edge_index[1]] - pos[edge_index[0]] + torch.mm(cell_shifts.to(pos.dtype), cell)
        idx = edge_index
        if self.core_cutoff < self.cutoff:
            keep = torch.linalg.norm(vec.detach(), dim=-1) < self.core_cutoff
            idx = edge_index[:, keep]
            vec = vec[keep]
        node_energy = self.core(atomic_numbers, idx, vec)
        energy = node_energy.sum()
        grad = torch.autograd.grad([energy], [pos], allow_unused=True)[0]
        forces = torch.zeros_like(pos) if grad is None else -grad
        return {"total_energy": energy.reshape(1), "node_energy": node_energy, "forces": forces}


def _example(model: nn.Module, dtype: torch.dtype, device):
    from ..data import structure_to_graph, synthetic
    species = list(getattr(model, "species", []) or [1, 6, 8])
    s = synthetic.organic_molecules(1, seed=11, labels=False)[0]
    z = torch.tensor(species)[torch.arange(s["atomic_numbers"].shape[0]) % len(species)]
    s["atomic_numbers"] = z
    g = structure_to_graph(s, float(model.cutoff))
    return (g.atomic_numbers.to(device), g.edge_index.to(device), g.edge_vectors().to(device, dtype))


def _core_model(model: nn.Module) -> nn.Module:
    inner = getattr(model, "model", None)
    if inner is not None and hasattr(model, "compute_forces"):
        model = inner
    if not hasattr(model, "node_energy"):
        raise TypeError(f"{type(model).__name__} has no node_energy(atomic_numbers, edge_index, edge_vec) core")
    return model


def deactivate_fast_paths(model: nn.Module) -> None:
    for m in model.modules():
        if hasattr(m, "set_use_fast"):
            m.set_use_fast(False)


def script_model(model: nn.Module, cutoff: Optional[float] = None) -> torch.jit.ScriptModule:
    """The scripted LAMMPS wrapper of ``model`` (fused kernels off inside the archive)."""
    core_model = _core_model(model)
    deactivate_fast_paths(core_model)
    dtype = next((p.dtype for p in core_model.parameters() if p.is_floating_point()), torch.get_default_dtype())
    device = next((p.device for p in core_model.parameters()), torch.device("cpu"))
    example = _example(core_model, dtype, device)
    with torch.no_grad():
        traced = torch.jit.trace(_EnergyCore(core_model).eval(), example, check_trace=False)
    cut = float(cutoff if cutoff is not None else core_model.cutoff)
    return torch.jit.script(LAMMPSWrapper(traced, cut, float(core_model.cutoff)).eval())


def export_to_lammps(model: nn.Module, cutoff: Optional[float], path: str, metadata: Optional[dict] = None) -> str:
    """Save the scripted wrapper of ``model`` at ``path`` (cutoff and metadata as extra files)."""
    scripted = script_model(model, cutoff)
    extra = {"cutoff": str(scripted.cutoff)}
    species = getattr(_core_model(model), "species", None)
    if species:
        extra["species"] = json.dumps([int(z) for z in species])
    for k, v in (metadata or {}).items():
        extra[str(k)] = str(v)
    torch.jit.save(scripted, path, _extra_files=extra)
    return path


def load_lammps(path: str, device: str = "cpu"):
    """The scripted module and its extra files (strings)."""
    extra = {"cutoff": "", "species": ""}
    mod = torch.jit.load(path, map_location=device, _extra_files=extra)
    return mod, extra
