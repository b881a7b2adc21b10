"""The one data object every model consumes: a structure or a batch of structures.

Field names, shapes and conventions are the reference's public contract
(``src/xnn/common/data/atomic_data.py:211-261``): ``edge_index`` is ``[src, dst]`` (the
energy of ``dst`` depends on ``src``), ``cell_shifts`` are integer image shifts, the
edge vector is ``pos[dst] - pos[src] + cell_shifts @ cell`` (``:371-418``), ``cell`` rows
are lattice vectors, and ``compute_dtype`` lets a float64 geometry drive a float32 model.
"""
from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Optional

import torch
from torch import Tensor


@dataclass
class AtomicGraph:
    pos: Tensor
    atomic_numbers: Tensor
    edge_index: Tensor
    cell_shifts: Tensor
    batch: Tensor
    n_atoms: Tensor
    cell: Optional[Tensor] = None
    pbc: Optional[Tensor] = None
    energy: Optional[Tensor] = None
    forces: Optional[Tensor] = None
    stress: Optional[Tensor] = None
    energy_mask: Optional[Tensor] = None
    forces_mask: Optional[Tensor] = None
    stress_mask: Optional[Tensor] = None
    dipole: Optional[Tensor] = None
    polarizability: Optional[Tensor] = None
    dipole_mask: Optional[Tensor] = None
    polarizability_mask: Optional[Tensor] = None
    charges: Optional[Tensor] = None
    charges_mask: Optional[Tensor] = None
    fragment_charges: Optional[Tensor] = None
    fragment_charges_mask: Optional[Tensor] = None
    external_potential: Optional[Tensor] = None
    total_charge: Optional[Tensor] = None
    spin_multiplicity: Optional[Tensor] = None
    weight: Optional[Tensor] = None
    head: Optional[Tensor] = None
    properties: Optional[Tensor] = None
    properties_mask: Optional[Tensor] = None
    state: Optional[Tensor] = None
    site_species: Optional[Tensor] = None
    site_occupancy: Optional[Tensor] = None
    energy_weight: Optional[Tensor] = None
    force_weight: Optional[Tensor] = None
    stress_weight: Optional[Tensor] = None
    atom_force_weight: Optional[Tensor] = None
    compute_dtype: Optional[torch.dtype] = None
    # "dst" when the edges are grouped by receiver in increasing order (what the
    # neighbour lists produce and collate keeps); lets the fused kernels skip a sort
    edge_order: Optional[str] = None
    # the edges' CSR views packed as int64 ``[dst_ptr (N+1) | src_ptr (N+1) | src_perm (E)]``,
    # computed on the host by the padded collate so the device builds no plan per step; only
    # valid for this graph as it is (subsets and concatenations drop it)
    edge_plan: Optional[Tensor] = None

    # --- sizes -------------------------------------------------------------------
    @property
    def model_dtype(self) -> torch.dtype:
        return self.compute_dtype if self.compute_dtype is not None else self.pos.dtype

    @property
    def num_graphs(self) -> int:
        return int(self.n_atoms.shape[0])

    @property
    def num_nodes(self) -> int:
        return int(self.pos.shape[0])

    @property
    def num_edges(self) -> int:
        return int(self.edge_index.shape[1])

    # --- movement ----------------------------------------------------------------
    def to(self, device, non_blocking: bool = False) -> "AtomicGraph":
        kw = {}
        for f in fields(self):
            v = getattr(self, f.name)
            kw[f.name] = v.to(device, non_blocking=non_blocking) if isinstance(v, Tensor) else v
        return AtomicGraph(**kw)

    def pin_memory(self) -> "AtomicGraph":
        kw = {}
        for f in fields(self):
            v = getattr(self, f.name)
            kw[f.name] = v.pin_memory() if isinstance(v, Tensor) else v
        return AtomicGraph(**kw)

    def clone(self) -> "AtomicGraph":
        kw = {}
        for f in fields(self):
            v = getattr(self, f.name)
            kw[f.name] = v.clone() if isinstance(v, Tensor) else v
        return AtomicGraph(**kw)

    def nbytes(self) -> int:
        return sum(v.numel() * v.element_size() for f in fields(self)
                   if isinstance(v := getattr(self, f.name), Tensor))

    # --- subsets -----------------------------------------------------------------
    def subset(self, keep: Tensor) -> "AtomicGraph":
        """The structures flagged in ``keep`` (``(B,)`` bool) as their own batch."""
        keep = keep.to(device=self.batch.device, dtype=torch.bool)
        node_keep = keep[self.batch]
        edge_keep = node_keep[self.edge_index[0]]
        new_node = torch.cumsum(node_keep.long(), 0) - 1
        new_graph = torch.cumsum(keep.long(), 0) - 1
        per_node = {"forces", "charges", "fragment_charges", "external_potential",
                    "site_species", "site_occupancy", "atom_force_weight"}
        kw = dict(pos=self.pos[node_keep], atomic_numbers=self.atomic_numbers[node_keep],
                  edge_index=new_node[self.edge_index[:, edge_keep]],
                  cell_shifts=self.cell_shifts[edge_keep],
                  batch=new_graph[self.batch[node_keep]], n_atoms=self.n_atoms[keep],
                  compute_dtype=self.compute_dtype, edge_order=self.edge_order, edge_plan=None)
        for f in fields(self):
            if f.name in kw:
                continue
            v = getattr(self, f.name)
            if isinstance(v, Tensor):
                m = node_keep if f.name in per_node else keep
                kw[f.name] = v[m.to(v.device)]
        return AtomicGraph(**kw)

    # --- geometry ----------------------------------------------------------------
    def edge_vectors(self) -> Tensor:
        """``pos[dst] - pos[src] + cell_shifts @ cell`` per edge, in :attr:`model_dtype`.

        Formed in the geometry dtype and only then rounded to the model dtype, so a
        float64 geometry driving a float32 model loses nothing to large coordinates.
        Differentiable with respect to ``pos`` and ``cell``.
        """
        src, dst = self.edge_index[0], self.edge_index[1]
        vec = self.pos.index_select(0, dst) - self.pos.index_select(0, src)
        if self.cell is not None:
            shifts = self.cell_shifts.to(vec.dtype)
            if self.cell.shape[0] == 1:
                vec = vec + shifts @ self.cell[0].to(vec.dtype)
            else:
                cell_e = self.cell.to(vec.dtype).index_select(0, self.batch.index_select(0, src))
                vec = vec + torch.einsum("ei,eij->ej", shifts, cell_e)
        return vec.to(self.model_dtype)
