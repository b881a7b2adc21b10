"""Captured evaluation: a model's energy/forces/stress replayed as one CUDA graph.

Behaviour follows the reference's ``GraphedEvaluation`` (``src/xnn/common/deploy/graphed_eval.py:44``):
structures are padded to fixed capacities with an inert padding structure plus headroom
(5 %), the evaluation is captured once and replayed; a structure that outgrows the capacities
triggers a new capture. On small systems an evaluation is bound by kernel launches, which the
replay removes.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
from torch import Tensor, nn

from ..data.atomic_graph import AtomicGraph
from ..train.graphed import GraphedStep, pad_graph


class GraphedEvaluation:
    def __init__(self, model: nn.Module, headroom: float = 0.05):
        self.model = model
        self.headroom = float(headroom)
        self._step: Optional[GraphedStep] = None
        self._cap = (0, 0, 0)
        self.captures = 0

    def _fits(self, g: AtomicGraph) -> bool:
        n, e, b = self._cap
        return g.num_nodes + 1 <= n and g.num_edges <= e and g.num_graphs + 1 <= b

    def _capture(self, g: AtomicGraph) -> None:
        h = 1.0 + self.headroom
        self._cap = (int(g.num_nodes * h) + 2, int(g.num_edges * h) + 1, g.num_graphs + 1)
        if self._step is not None:
            self._step.release()
        padded = self._pad(g)
        self._step = GraphedStep(lambda b: self.model(b), padded, g.pos.device)
        self.captures += 1

    def _pad(self, g: AtomicGraph) -> AtomicGraph:
        cutoff = float(getattr(self.model, "cutoff", 5.0) or 5.0)
        return pad_graph(g, *self._cap, cutoff)

    def __call__(self, g: AtomicGraph) -> Dict[str, Tensor]:
        if self._step is None or not self._fits(g):
            self._capture(g)
        out = self._step(self._pad(g))
        n, b = g.num_nodes, g.num_graphs
        res: Dict[str, Tensor] = {}
        for k, v in out.items():
            if not torch.is_tensor(v) or v.dim() == 0:
                continue
            if v.shape[0] == self._cap[0]:
                res[k] = v[:n].clone()
            elif v.shape[0] == self._cap[2]:
                res[k] = v[:b].clone()
        return res

    def release(self) -> None:
        if self._step is not None:
            self._step.release()
            self._step = None
