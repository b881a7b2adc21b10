"""Molecular-dynamics steps replayed as one CUDA graph on a Verlet skin list.

:class:`StepGraph` evaluates energy, forces (and stress) of a moving structure. The pair list is
built once with ``cutoff + skin`` and kept while every atom stays within half the skin of where it
was at the build (minimum image in a cell, the cell unchanged); the list's capacity is ``margin``
times its first length, so a rebuild refreshes the padded buffers in place and only a list that
outgrows the capacity re-records. After ``warmup`` eager steps the evaluation is captured once on a
GPU and replayed each step (one launch instead of hundreds: small systems are launch bound).

Skin lists need pair terms that vanish beyond the cutoff, which every model here has (envelopes
that are exactly zero past ``r_c``; the classical force fields mask their pair sums at the cutoff).
Padding: a fixed-topology force field takes copies of one of its excluded pairs (weighted out by
the exclusion mask, no extra atoms); any other model takes an inert padding structure
(:func:`xnn_b200.train.graphed.pad_graph`).

:class:`VerletStepper` integrates velocity Verlet on a :class:`StepGraph` (the reference's
``ClassicalStepper`` / ``ReaxFFStepper`` role: skin lists, kernels only, graph replay). Behaviour
follows the reference's ``src/xnn/common/deploy/step_graph.py:49`` and
``src/xnn/ffnn/models/classical_step.py:63``.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..data.neighborlist import build_neighbor_list
from ..models.outputs import ForceStressOutput
from ..train.graphed import GraphedStep, pad_graph

EV_A2_AMU_TO_A_FS2 = 9.648533212331e-3          # eV / (Å amu) in Å / fs^2


def _core(model: nn.Module) -> nn.Module:
    return getattr(model, "model", model)


class StepGraph:
    """``step(struct) -> {"energy", "forces"[, "stress"]}`` for one structure ``{"pos",
    "atomic_numbers"[, "cell", "pbc"]}`` of fixed size."""

    def __init__(self, model: nn.Module, cutoff: Optional[float] = None, skin: float = 1.0, margin: float = 1.2,
                 warmup: int = 2, compute_stress: bool = False, capture: Optional[bool] = None):
        self.model = model
        self.cutoff = float(cutoff if cutoff is not None else getattr(_core(model), "cutoff"))
        self.skin, self.margin, self.warmup = float(skin), float(margin), int(warmup)
        self.compute_stress = bool(compute_stress)
        self.capture = capture
        self.out_model = ForceStressOutput(model, compute_stress=compute_stress)
        self.topology_padding = hasattr(_core(model), "excl_index") and _core(model).excl_index.shape[1] > 0
        self.reset()

    def reset(self) -> None:
        self._ref_pos = self._cell = None
        self._edges = self._shifts = None
        self._capacity = 0
        self._graphed: Optional[GraphedStep] = None
        self.steps = self.rebuilds = self.captures = 0

    # ------------------------------------------------------------------------------- pair list
    def _needs_rebuild(self, pos: Tensor, cell: Optional[Tensor]) -> bool:
        if self._ref_pos is None:
            return True
        if (cell is None) != (self._cell is None) or (cell is not None and not torch.equal(cell, self._cell)):
            return True
        d = pos - self._ref_pos
        if cell is not None:
            frac = d @ torch.linalg.inv(cell)
            d = (frac - torch.round(frac)) @ cell
        return bool((d * d).sum(1).max() > (0.5 * self.skin) ** 2) if len(d) else False

    def _rebuild(self, pos: Tensor, cell: Optional[Tensor], pbc: Optional[Tensor]) -> None:
        ei, sh = build_neighbor_list(pos.detach(), self.cutoff + self.skin, cell, pbc)
        self._edges, self._shifts = ei, sh
        self._ref_pos, self._cell = pos.detach().clone(), None if cell is None else cell.detach().clone()
        self.rebuilds += 1
        if ei.shape[1] > self._capacity:
            self._capacity = max(int(ei.shape[1] * self.margin) + 1, 1)
            if self._graphed is not None:
                self._graphed.release()
                self._graphed = None

    def _graph(self, struct: dict) -> AtomicGraph:
        pos = struct["pos"]
        n, dev = pos.shape[0], pos.device
        cell, pbc = struct.get("cell"), struct.get("pbc")
        ei, sh = self._edges, self._shifts
        pad = self._capacity - ei.shape[1]
        kw = dict(pos=pos, atomic_numbers=struct["atomic_numbers"].to(dev), batch=torch.zeros(n, dtype=torch.long, device=dev),
                  n_atoms=torch.tensor([n], device=dev))
        if cell is not None:
            kw["cell"], kw["pbc"] = cell.reshape(1, 3, 3), (pbc if pbc is not None else torch.ones(3, dtype=torch.bool,
                                                                                                   device=dev)).reshape(1, 3)
        if self.topology_padding:
            # copies of an excluded pair contribute nothing
            ex = _core(self.model).excl_index[:, :1].to(dev)
            ei = torch.cat([ei, ex.expand(2, pad)], 1)
            sh = torch.cat([sh, sh.new_zeros(pad, 3)])
            return AtomicGraph(edge_index=ei, cell_shifts=sh, **kw)
        g = AtomicGraph(edge_index=ei, cell_shifts=sh, **kw)
        return pad_graph(g, n + 2, self._capacity, 2, self.cutoff)

    # ------------------------------------------------------------------------------ evaluation
    def _want_capture(self, dev) -> bool:
        if self.capture is not None:
            return bool(self.capture)
        return dev.type == "cuda" and bool(getattr(_core(self.model), "graph_capturable", True))

    def __call__(self, struct: dict) -> Dict[str, Tensor]:
        pos = struct["pos"]
        cell = struct.get("cell")
        cell = None if cell is None else cell.reshape(3, 3)
        if self._needs_rebuild(pos.detach(), cell):
            self._rebuild(pos, cell, struct.get("pbc"))
        g = self._graph(struct)
        n = pos.shape[0]
        self.steps += 1
        if self._want_capture(pos.device) and self.steps > self.warmup:
            if self._graphed is None:
                self._graphed = GraphedStep(self.out_model, g, pos.device)
                self.captures += 1
            out = self._graphed(g)
        else:
            out = self.out_model(g)
        res = {"energy": out["energy"][:1].detach(), "forces": out["forces"][:n].detach()}
        if self.compute_stress and "stress" in out:
            res["stress"] = out["stress"][:1].detach()
        return res

    def release(self) -> None:
        if self._graphed is not None:
            self._graphed.release()
            self._graphed = None


class VerletStepper:
    """Velocity Verlet on a :class:`StepGraph` (positions Å, velocities Å/fs, masses amu, dt fs)."""

    def __init__(self, step_graph: StepGraph, struct: dict, masses: Tensor, dt: float = 0.5,
                 velocities: Optional[Tensor] = None):
        self.sg, self.struct, self.dt = step_graph, dict(struct), float(dt)
        self.masses = masses.to(struct["pos"])
        self.vel = torch.zeros_like(struct["pos"]) if velocities is None else velocities.to(struct["pos"]).clone()
        self.out = self.sg(self.struct)

    def step(self) -> Dict[str, Tensor]:
        acc = self.out["forces"] / self.masses[:, None] * EV_A2_AMU_TO_A_FS2
        self.vel = self.vel + 0.5 * self.dt * acc
        self.struct["pos"] = self.struct["pos"] + self.dt * self.vel
        self.out = self.sg(self.struct)
        self.vel = self.vel + 0.5 * self.dt * self.out["forces"] / self.masses[:, None] * EV_A2_AMU_TO_A_FS2
        return self.out

    def kinetic_energy(self) -> Tensor:
        return 0.5 * (self.masses[:, None] * self.vel * self.vel).sum() / EV_A2_AMU_TO_A_FS2

    def run(self, n_steps: int) -> Dict[str, Tensor]:
        for _ in range(int(n_steps)):
            self.step()
        return self.out
