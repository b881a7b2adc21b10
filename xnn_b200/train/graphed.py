"""Fixed-shape batches and training steps replayed as one CUDA graph.

A captured step needs the same tensor shapes every time. :class:`PaddedCollate` pads a
batch to fixed atom / edge / structure capacities with inert padding
(``src/xnn/common/train/graphed.py:235``): padding atoms sit on a line ``2.5 cutoff``
apart in a dummy structure whose labels are masked out, and every padding edge joins
two neighbouring padding atoms, so it lies outside the cutoff and contributes exactly
zero to every sum and derivative. Receivers of padding edges are spread over the padding
atoms so the per-atom kernels see no long tail, and the edges stay grouped by receiver.

:class:`GraphedStep` warms a step function up on a side stream, captures it once, and
afterwards copies each padded batch into the captured input buffers and replays the
graph: the forward, the force pass, the loss, the double backward, the gradient all-reduce
and the optimizer update run as one launch.
"""
from __future__ import annotations

from dataclasses import fields
from typing import Callable, Iterable, Optional

import torch
from torch import Tensor

from ..data import AtomicGraph, collate

_PER_NODE = {"forces", "charges", "fragment_charges", "external_potential", "site_species",
             "site_occupancy", "atom_force_weight"}


def batch_sizes(graphs: Iterable[AtomicGraph]):
    n = e = b = 0
    for g in graphs:
        n += g.num_nodes
        e += g.num_edges
        b += g.num_graphs
    return n, e, b


class PaddedCollate:
    """Collate and pad to ``(max_atoms, max_edges, max_graphs)`` (see module notes)."""

    def __init__(self, max_atoms: int, max_edges: int, max_graphs: int, cutoff: float,
                 pin_memory: bool = False):
        self.max_atoms = int(max_atoms)
        self.max_edges = int(max_edges)
        self.max_graphs = int(max_graphs)
        self.cutoff = float(cutoff)
        self.pin_memory = pin_memory

    def fits(self, graphs) -> bool:
        n, e, b = batch_sizes(graphs)
        return n + 2 <= self.max_atoms and e <= self.max_edges and b + 1 <= self.max_graphs

    def __call__(self, graphs) -> AtomicGraph:
        b = collate(list(graphs))
        out = pad_graph(b, self.max_atoms, self.max_edges, self.max_graphs, self.cutoff)
        return out.pin_memory() if self.pin_memory else out


def pad_graph(b: AtomicGraph, max_atoms: int, max_edges: int, max_graphs: int, cutoff: float) -> AtomicGraph:
    n, e, B = b.num_nodes, b.num_edges, b.num_graphs
    if n + 2 > max_atoms or e > max_edges or B + 1 > max_graphs:
        raise ValueError(f"batch ({n} atoms, {e} edges, {B} structures) exceeds the capacity "
                         f"({max_atoms}, {max_edges}, {max_graphs - 1})")
    dev = b.pos.device
    na, ne, nb = max_atoms - n, max_edges - e, max_graphs - B
    pad_struct = max_graphs - 1
    far = float(b.pos.detach().abs().max()) + 10.0 * cutoff if n else 0.0
    xs = far + 2.5 * cutoff * torch.arange(na, dtype=b.pos.dtype, device=dev)
    pad_pos = torch.stack([xs, torch.zeros_like(xs), torch.zeros_like(xs)], 1)
    # padding edges: receivers spread over the padding atoms (non-decreasing), sender next to it
    k = torch.arange(ne, device=dev)
    dst_local = (k * na) // max(ne, 1)
    src_local = torch.where(dst_local + 1 < na, dst_local + 1, dst_local - 1)
    pad_edges = torch.stack([src_local + n, dst_local + n])
    kw = dict(
        pos=torch.cat([b.pos.detach(), pad_pos]),
        atomic_numbers=torch.cat([b.atomic_numbers, b.atomic_numbers.new_full((na,), int(b.atomic_numbers[0]) if n else 1)]),
        edge_index=torch.cat([b.edge_index, pad_edges], 1),
        cell_shifts=torch.cat([b.cell_shifts, b.cell_shifts.new_zeros(ne, 3)]),
        batch=torch.cat([b.batch, b.batch.new_full((na,), pad_struct)]),
        n_atoms=torch.cat([b.n_atoms, b.n_atoms.new_ones(nb - 1), b.n_atoms.new_tensor([na])]),
        compute_dtype=b.compute_dtype, edge_order=b.edge_order,
    )
    if b.cell is not None:
        kw["cell"] = torch.cat([b.cell, b.cell.new_zeros(nb, 3, 3)])
        kw["pbc"] = torch.cat([b.pbc.to(dev), torch.zeros(nb, 3, dtype=torch.bool, device=dev)])
    ones_b = torch.ones(B, dtype=torch.bool, device=dev)
    zeros_nb = torch.zeros(nb, dtype=torch.bool, device=dev)
    masks = {"energy": "energy_mask", "forces": "forces_mask", "stress": "stress_mask",
             "dipole": "dipole_mask", "polarizability": "polarizability_mask",
             "charges": "charges_mask", "properties": "properties_mask"}
    for f in fields(AtomicGraph):
        name = f.name
        if name in kw or name in ("cell", "pbc", "edge_plan") or name.endswith("_mask"):
            continue
        v = getattr(b, name)
        if not isinstance(v, Tensor):
            continue
        rows = na if name in _PER_NODE else nb
        kw[name] = torch.cat([v, v.new_zeros((rows,) + tuple(v.shape[1:]))])
        if name in masks:
            m = getattr(b, masks[name])
            kw[masks[name]] = torch.cat([m if m is not None else ones_b, zeros_nb])
    afw = b.atom_force_weight if b.atom_force_weight is not None else b.pos.new_ones(n)
    kw["atom_force_weight"] = torch.cat([afw, afw.new_zeros(na)])
    kw["edge_plan"] = packed_edge_plan(kw["edge_index"], max_atoms)
    return AtomicGraph(**kw)


def packed_edge_plan(edge_index: Tensor, n_nodes: int) -> Tensor:
    """``[dst_ptr | src_ptr | src_perm]`` (int64) of receiver-sorted edges, on the host."""
    import numpy as np
    ei = edge_index.detach().cpu().numpy()
    src, dst = ei[0], ei[1]
    dst_ptr = np.zeros(n_nodes + 1, dtype=np.int64)
    np.cumsum(np.bincount(dst, minlength=n_nodes), out=dst_ptr[1:])
    src_ptr = np.zeros(n_nodes + 1, dtype=np.int64)
    np.cumsum(np.bincount(src, minlength=n_nodes), out=src_ptr[1:])
    src_perm = np.argsort(src, kind="stable").astype(np.int64)
    return torch.from_numpy(np.concatenate([dst_ptr, src_ptr, src_perm])).to(edge_index.device)


def copy_graph_(dst: AtomicGraph, src: AtomicGraph) -> None:
    """Copy every tensor of ``src`` into the same-shaped tensor of ``dst`` (non-blocking)."""
    for f in fields(AtomicGraph):
        a = getattr(dst, f.name)
        b = getattr(src, f.name)
        if isinstance(a, Tensor):
            if not isinstance(b, Tensor) or a.shape != b.shape:
                raise ValueError(f"field {f.name}: captured {tuple(a.shape)}, got "
                                 f"{None if b is None else tuple(b.shape)}")
            with torch.no_grad():
                a.copy_(b, non_blocking=True)


class GraphedStep:
    """One training (or evaluation) step captured as a CUDA graph over static inputs."""

    def __init__(self, step: Callable[[AtomicGraph], object], example: AtomicGraph,
                 device: torch.device, warmup: int = 3):
        self.step = step
        self.static = example.to(device)
        self.static.pos.requires_grad_(False)
        s = torch.cuda.Stream(device=device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._run()
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = self._run()

    def _run(self):
        g = AtomicGraph(**{f.name: getattr(self.static, f.name) for f in fields(AtomicGraph)})
        return self.step(g)

    def __call__(self, batch: AtomicGraph):
        copy_graph_(self.static, batch)
        self.graph.replay()
        return self.out

    def release(self) -> None:
        self.graph.reset()
        self.graph = None
