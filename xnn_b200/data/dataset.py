"""Structures to graphs, datasets and batching.

``structure_to_graph`` turns a structure dict (``pos``, ``atomic_numbers``, optional
``cell``/``pbc`` and labels) into an :class:`AtomicGraph`; ``collate`` concatenates
graphs, offsets the edge indices and masks missing labels so molecules and cells,
and structures with different label sets, share one batch
(``src/xnn/common/data/dataset.py:21,245,371``). Energies are float64.
"""
from __future__ import annotations

from dataclasses import fields
from typing import Callable, Dict, List, Optional, Sequence

import torch
from torch import Tensor

from .atomic_graph import AtomicGraph
from .neighborlist import build_neighbor_list

_PER_NODE = {"forces", "charges", "fragment_charges", "external_potential", "site_species",
             "site_occupancy", "atom_force_weight"}
_MASKED = {"energy": "energy_mask", "forces": "forces_mask", "stress": "stress_mask",
           "dipole": "dipole_mask", "polarizability": "polarizability_mask",
           "charges": "charges_mask", "properties": "properties_mask",
           "fragment_charges": "fragment_charges_mask"}


def structure_to_graph(s: Dict, cutoff: float, device=None, max_neighbors: Optional[int] = None,
                       engine: str = "auto") -> AtomicGraph:
    """Build a single-structure graph; see the module notes for the accepted keys."""
    fdt = torch.get_default_dtype()

    def t(x, dtype=fdt):
        return torch.as_tensor(x, dtype=dtype, device=device)

    pos = t(s["pos"], s["pos"].dtype if isinstance(s["pos"], Tensor) and s["pos"].is_floating_point() else fdt)
    z = torch.as_tensor(s["atomic_numbers"], dtype=torch.long, device=device)
    cell = s.get("cell")
    pbc = s.get("pbc")
    if cell is not None:
        cell = t(cell, pos.dtype).reshape(3, 3)
        pbc = torch.ones(3, dtype=torch.bool) if pbc is None else torch.as_tensor(pbc, dtype=torch.bool)
    else:
        pbc = None
    edge_index, shifts = build_neighbor_list(pos, cutoff, cell, pbc, engine=engine)
    if max_neighbors is not None:
        from .neighborlist import nearest_edges
        vec = pos[edge_index[1]] - pos[edge_index[0]]
        if cell is not None:
            vec = vec + shifts.to(pos.dtype) @ cell
        keep = nearest_edges(edge_index, vec.norm(dim=-1), max_neighbors, pos.shape[0])
        edge_index, shifts = edge_index[:, keep], shifts[keep]
    n = pos.shape[0]
    g = AtomicGraph(pos=pos, atomic_numbers=z, edge_index=edge_index.to(device),
                    cell_shifts=shifts.to(device),
                    batch=torch.zeros(n, dtype=torch.long, device=device),
                    n_atoms=torch.tensor([n], dtype=torch.long, device=device),
                    cell=None if cell is None else cell[None],
                    pbc=None if pbc is None else pbc[None], edge_order="dst")
    if "energy" in s and s["energy"] is not None:
        g.energy = torch.as_tensor([float(s["energy"])], dtype=torch.float64, device=device)
    if "forces" in s and s["forces"] is not None:
        g.forces = t(s["forces"]).reshape(n, 3)
    if "stress" in s and s["stress"] is not None:
        g.stress = t(s["stress"]).reshape(1, 3, 3)
    for key in ("dipole", "dipole_moment"):
        if key in s and s[key] is not None:
            g.dipole = t(s[key]).reshape(1, 3)
    if "polarizability" in s and s["polarizability"] is not None:
        g.polarizability = t(s["polarizability"]).reshape(1, 3, 3)
    if "charges" in s and s["charges"] is not None:
        g.charges = t(s["charges"]).reshape(n)
    for key in ("total_charge", "charge"):
        if key in s and s[key] is not None:
            g.total_charge = t([float(s[key])])
    for key in ("spin_multiplicity", "multiplicity"):
        if key in s and s[key] is not None:
            g.spin_multiplicity = t([float(s[key])])
    for key in ("weight", "energy_weight", "force_weight", "stress_weight"):
        if key in s and s[key] is not None:
            setattr(g, key, t([float(s[key])]))
    if "head" in s and s["head"] is not None:
        g.head = torch.as_tensor([int(s["head"])], dtype=torch.long, device=device)
    if "properties" in s and s["properties"] is not None:
        g.properties = t(s["properties"]).reshape(1, -1)
    if "atom_force_weight" in s and s["atom_force_weight"] is not None:
        g.atom_force_weight = t(s["atom_force_weight"]).reshape(n)
    return g


def collate(graphs: Sequence[AtomicGraph]) -> AtomicGraph:
    """Concatenate graphs into one batch (edge indices offset, missing labels masked)."""
    if len(graphs) == 1 and graphs[0].num_graphs == 1:
        return graphs[0]
    pos = torch.cat([g.pos for g in graphs])
    device = pos.device
    counts = torch.tensor([g.num_nodes for g in graphs], dtype=torch.long)
    offsets = torch.cumsum(counts, 0) - counts
    edge_index = torch.cat([g.edge_index + int(o) for g, o in zip(graphs, offsets)], dim=1)
    batch_sizes = [g.num_graphs for g in graphs]
    batch_offsets = torch.cumsum(torch.tensor(batch_sizes), 0) - torch.tensor(batch_sizes)
    batch = torch.cat([g.batch + int(o) for g, o in zip(graphs, batch_offsets)])
    out = dict(pos=pos, atomic_numbers=torch.cat([g.atomic_numbers for g in graphs]),
               edge_index=edge_index, cell_shifts=torch.cat([g.cell_shifts for g in graphs]),
               batch=batch, n_atoms=torch.cat([g.n_atoms for g in graphs]),
               compute_dtype=graphs[0].compute_dtype,
               edge_order="dst" if all(g.edge_order == "dst" for g in graphs) else None)
    if any(g.cell is not None for g in graphs):
        out["cell"] = torch.cat([g.cell if g.cell is not None else
                                 pos.new_zeros(g.num_graphs, 3, 3) for g in graphs])
        out["pbc"] = torch.cat([g.pbc.to(device) if g.pbc is not None else
                                torch.zeros(g.num_graphs, 3, dtype=torch.bool, device=device)
                                for g in graphs])
    skip = set(out) | {"cell", "pbc"} | set(_MASKED.values())
    for f in fields(AtomicGraph):
        name = f.name
        if name in skip or name in ("compute_dtype", "edge_order", "edge_plan"):
            continue
        vals = [getattr(g, name) for g in graphs]
        if all(v is None for v in vals):
            continue
        ref = next(v for v in vals if v is not None)
        filled, mask = [], []
        for g, v in zip(graphs, vals):
            rows = g.num_nodes if name in _PER_NODE else g.num_graphs
            if v is None:
                filled.append(torch.zeros((rows,) + tuple(ref.shape[1:]), dtype=ref.dtype, device=ref.device))
                mask.append(torch.zeros(g.num_graphs, dtype=torch.bool, device=device))
            else:
                filled.append(v)
                m = getattr(g, _MASKED[name]) if name in _MASKED else None
                mask.append(m if m is not None else torch.ones(g.num_graphs, dtype=torch.bool, device=device))
        out[name] = torch.cat(filled)
        if name in _MASKED and not all(bool(m.all()) for m in mask):
            out[_MASKED[name]] = torch.cat(mask)
    return AtomicGraph(**out)


class AtomicDataset(torch.utils.data.Dataset):
    """A list of structure dicts turned into graphs once (cached per index)."""

    def __init__(self, structures: List[Dict], cutoff: float, transform: Optional[Callable] = None,
                 max_neighbors: Optional[int] = None, precompute: bool = False):
        self.structures = list(structures)
        self.cutoff = float(cutoff)
        self.transform = transform
        self.max_neighbors = max_neighbors
        self._cache: Dict[int, AtomicGraph] = {}
        if precompute:
            for i in range(len(self)):
                self[i]

    @classmethod
    def from_file(cls, path: str, cutoff: float, **kwargs) -> "AtomicDataset":
        from .io import read_structures
        return cls(read_structures(path, **{k: v for k, v in kwargs.items()
                                            if k in ("energy_key", "forces_key", "stress_key")}),
                   cutoff, **{k: v for k, v in kwargs.items()
                              if k not in ("energy_key", "forces_key", "stress_key")})

    def __len__(self) -> int:
        return len(self.structures)

    def __getitem__(self, i: int) -> AtomicGraph:
        g = self._cache.get(i)
        if g is None:
            g = structure_to_graph(self.structures[i], self.cutoff, max_neighbors=self.max_neighbors)
            self._cache[i] = g
        return self.transform(g) if self.transform is not None else g
