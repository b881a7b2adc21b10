"""Self-contained TorchScript archives and the OpenMM-style force module.

``export_torchscript(model, path)`` saves a module with two entry points, as the reference's
``src/xnn/common/deploy/torchscript.py:618-924`` does: ``forward(pos, atomic_numbers, cell, pbc)``
builds its own neighbour list (a scripted all-pairs search over the periodic images) and returns
energy, forces and, for a periodic cell, the stress; ``forward_lammps(pos, edge_index,
cell_shifts, atomic_numbers, cell)`` takes host-built neighbour data. The model core is traced
with the fused kernels off (see :mod:`xnn_b200.deploy.lammps`).

:class:`OpenMMForce` is the ``TorchForce`` contract of openmm-torch: ``forward(positions)`` in nm
(and optionally the box vectors in nm) returning the energy in kJ/mol for a fixed list of atomic
numbers; it works without OpenMM installed (it is a plain scripted module).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch
from torch import Tensor, nn

from .lammps import _core_model, _EnergyCore, _example, deactivate_fast_paths

EV_TO_KJ_MOL = 96.48533212331002


@torch.jit.script
def neighbor_list_ts(pos: Tensor, cutoff: float, cell: Tensor, pbc: Tensor) -> Tuple[Tensor, Tensor]:
    """Edges ``[src, dst]`` within ``cutoff`` (periodic images along ``pbc`` axes) and their
    integer cell shifts, with ``vec = pos[dst] - pos[src] + shift @ cell``."""
    n = pos.shape[0]
    reps: List[int] = [0, 0, 0]
    if bool(pbc.any()):
        vol = torch.abs(torch.det(cell))
        for a in range(3):
            if bool(pbc[a]):
                b = cell[(a + 1) % 3]
                c = cell[(a + 2) % 3]
                h = vol / torch.linalg.norm(torch.linalg.cross(b, c))
                reps[a] = int(math.ceil(cutoff / float(h)))
    rx = torch.arange(-reps[0], reps[0] + 1, device=pos.device)
    ry = torch.arange(-reps[1], reps[1] + 1, device=pos.device)
    rz = torch.arange(-reps[2], reps[2] + 1, device=pos.device)
    shifts = torch.cartesian_prod(rx, ry, rz).reshape(-1, 3)
    disp = shifts.to(pos.dtype) @ cell
    src_l: List[Tensor] = []
    dst_l: List[Tensor] = []
    sh_l: List[Tensor] = []
    for k in range(shifts.shape[0]):
        d = pos[None, :, :] - pos[:, None, :] + disp[k]          # [i, j]: pos[j] - pos[i] + shift
        within = (d * d).sum(-1) < cutoff * cutoff
        if bool((shifts[k] == 0).all()):
            within = within & ~torch.eye(n, dtype=torch.bool, device=pos.device)
        ij = torch.nonzero(within)
        dst_l.append(ij[:, 0])
        src_l.append(ij[:, 1])
        sh_l.append(shifts[k].expand(ij.shape[0], 3))
    edge_index = torch.stack([torch.cat(src_l), torch.cat(dst_l)])
    # the edge vector pos[dst] - pos[src] + S @ cell equals pos[i] - pos[j] - shift: S = -shift
    return edge_index, -torch.cat(sh_l)


class _Standalone(nn.Module):
    def __init__(self, core: nn.Module, cutoff: float):
        super().__init__()
        self.core = core
        self.cutoff = float(cutoff)

    def forward_lammps(self, pos: Tensor, edge_index: Tensor, cell_shifts: Tensor, atomic_numbers: Tensor,
                       cell: Tensor) -> Dict[str, Tensor]:
        pos = pos.detach().requires_grad_(True)
        vec = pos[edge_index[1]] - pos[edge_index[0]] + torch.mm(cell_shifts.to(pos.dtype), cell)
        node_energy = self.core(atomic_numbers, edge_index, vec)
        energy = node_energy.sum()
        grad = torch.autograd.grad([energy], [pos], allow_unused=True)[0]
        forces = torch.zeros_like(pos) if grad is None else -grad
        return {"total_energy": energy.reshape(1), "node_energy": node_energy, "forces": forces}

    def forward(self, pos: Tensor, atomic_numbers: Tensor, cell: Tensor, pbc: Tensor) -> Dict[str, Tensor]:
        periodic = bool(pbc.any())
        edge_index, shifts = neighbor_list_ts(pos.detach(), self.cutoff, cell, pbc)
        p = pos.detach().requires_grad_(True)
        strain = torch.zeros((3, 3), dtype=pos.dtype, device=pos.device).requires_grad_(True)
        sym = 0.5 * (strain + strain.transpose(0, 1))
        ps = p + p @ sym
        cs = cell + cell @ sym
        vec = ps[edge_index[1]] - ps[edge_index[0]] + torch.mm(shifts.to(pos.dtype), cs)
        node_energy = self.core(atomic_numbers, edge_index, vec)
        energy = node_energy.sum()
        grads = torch.autograd.grad([energy], [p, strain], allow_unused=True)
        gp = grads[0]
        gs = grads[1]
        out: Dict[str, Tensor] = {"energy": energy.reshape(1), "node_energy": node_energy,
                                  "forces": torch.zeros_like(p) if gp is None else -gp}
        if periodic and gs is not None:
            out["stress"] = (gs / torch.abs(torch.det(cell))).reshape(1, 3, 3)
        return out


def export_torchscript(model: nn.Module, path: str, metadata: Optional[dict] = None) -> str:
    core_model = _core_model(model)
    deactivate_fast_paths(core_model)
    dtype = next((p.dtype for p in core_model.parameters() if p.is_floating_point()), torch.get_default_dtype())
    device = next((p.device for p in core_model.parameters()), torch.device("cpu"))
    with torch.no_grad():
        traced = torch.jit.trace(_EnergyCore(core_model).eval(), _example(core_model, dtype, device),
                                 check_trace=False)
    mod = torch.jit.script(_Standalone(traced, float(core_model.cutoff)).eval())
    extra = {"cutoff": str(float(core_model.cutoff))}
    for k, v in (metadata or {}).items():
        extra[str(k)] = str(v)
    torch.jit.save(mod, path, _extra_files=extra)
    return path


class OpenMMForce(nn.Module):
    """``energy (kJ/mol) = f(positions (nm)[, box (nm)])`` for fixed atomic numbers."""

    def __init__(self, core: nn.Module, atomic_numbers: Tensor, cutoff: float, periodic: bool):
        super().__init__()
        self.core = core
        self.register_buffer("atomic_numbers", atomic_numbers.clone())
        self.cutoff = float(cutoff)
        self.periodic = bool(periodic)
        self.ev_to_kj = float(EV_TO_KJ_MOL)

    def forward(self, positions: Tensor, boxvectors: Optional[Tensor] = None) -> Tensor:
        pos = positions * 10.0
        if self.periodic and boxvectors is not None:
            cell = boxvectors * 10.0
            pbc = torch.ones(3, dtype=torch.bool, device=pos.device)
        else:
            cell = torch.zeros((3, 3), dtype=pos.dtype, device=pos.device)
            pbc = torch.zeros(3, dtype=torch.bool, device=pos.device)
        edge_index, shifts = neighbor_list_ts(pos.detach(), self.cutoff, cell, pbc)
        vec = pos[edge_index[1]] - pos[edge_index[0]] + torch.mm(shifts.to(pos.dtype), cell)
        return self.core(self.atomic_numbers, edge_index, vec).sum() * self.ev_to_kj


class OpenMMSubsetForce(nn.Module):
    """An :class:`OpenMMForce` on the ``atoms`` of a larger OpenMM system (ML/MM): the model sees
    those atoms' positions only; every other particle gets no force from it."""

    def __init__(self, inner: nn.Module, atoms: Tensor):
        super().__init__()
        self.inner = inner
        self.register_buffer("atoms", atoms.clone())

    def forward(self, positions: Tensor, boxvectors: Optional[Tensor] = None) -> Tensor:
        return self.inner(positions.index_select(0, self.atoms), boxvectors)


def openmm_force(model: nn.Module, atomic_numbers, periodic: bool = False, atoms=None) -> torch.jit.ScriptModule:
    """The scripted OpenMM force module (save it with ``torch.jit.save`` for ``TorchForce``); with
    ``atoms`` (indices into the OpenMM system) it acts on that subset of a larger system."""
    core_model = _core_model(model)
    deactivate_fast_paths(core_model)
    dtype = next((p.dtype for p in core_model.parameters() if p.is_floating_point()), torch.get_default_dtype())
    device = next((p.device for p in core_model.parameters()), torch.device("cpu"))
    with torch.no_grad():
        traced = torch.jit.trace(_EnergyCore(core_model).eval(), _example(core_model, dtype, device),
                                 check_trace=False)
    z = torch.as_tensor(atomic_numbers, dtype=torch.long, device=device)
    inner = OpenMMForce(traced, z, float(core_model.cutoff), periodic).eval()
    if atoms is not None:
        idx = torch.as_tensor(list(atoms), dtype=torch.long, device=device)
        if idx.numel() != z.numel():
            raise ValueError(f"{idx.numel()} atoms for {z.numel()} atomic numbers")
        return torch.jit.script(OpenMMSubsetForce(inner, idx).eval())
    return torch.jit.script(inner)
