"""Captured evaluation: a model's energy/forces/stress replayed as one CUDA graph.

Behaviour follows the reference's ``GraphedEvaluation`` (``src/xnn/common/deploy/graphed_eval.py:44``):
structures are padded to fixed capacities with an inert padding structure plus headroom
(5 %), the evaluation is captured once and replayed; a structure that outgrows the capacities
triggers a new capture. On small systems an evaluation is bound by kernel launches, which the
replay removes; on large ones the launches matter little and the padding costs more, so:

* the first inputs are evaluated ordinarily and timed (up to :data:`PROBES` of them); when none
  is faster than ``max_ms`` the evaluations stay ordinary and nothing is captured;
* after every capture ``trial`` replays are timed against ``trial`` ordinary evaluations
  (CUDA events, each bracketed by a synchronisation) and the faster is kept until the input
  outgrows the capacities; when the ordinary evaluation wins the graph and its memory are
  released.

The replay runs the same code as the ordinary evaluation, so the two agree to round-off. On a CPU
every evaluation is ordinary.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
from torch import Tensor, nn

from ..data.atomic_graph import AtomicGraph
from ..train.graphed import GraphedStep, pad_graph

#: ordinary evaluations timed at most before deciding that inputs are too large to capture
PROBES = 4


class GraphedEvaluation:
    def __init__(self, model: nn.Module, headroom: float = 0.05, trial: int = 3, max_ms: Optional[float] = 100.0):
        self.model = model
        self.headroom = float(headroom)
        self.trial = int(trial)
        self.max_ms = max_ms
        self._step: Optional[GraphedStep] = None
        self._cap = (0, 0, 0)
        self.captures = 0
        self.probes = 0
        self.capturable: Optional[bool] = None if max_ms is not None else True
        #: after a trial: whether the replay was the faster (evaluations then replay)
        self.replay = True
        self.trial_ms: Dict[str, float] = {}

    # ------------------------------------------------------------------ pieces
    def _fits(self, g: AtomicGraph) -> bool:
        n, e, b = self._cap
        return g.num_nodes + 1 <= n and g.num_edges <= e and g.num_graphs + 1 <= b

    def _capture(self, g: AtomicGraph) -> None:
        h = 1.0 + self.headroom
        self._cap = (int(g.num_nodes * h) + 2, int(g.num_edges * h) + 1, g.num_graphs + 1)
        self.release()
        padded = self._pad(g)
        self._step = GraphedStep(lambda b: self.model(b), padded, g.pos.device)
        self.captures += 1

    def _pad(self, g: AtomicGraph) -> AtomicGraph:
        cutoff = float(getattr(self.model, "cutoff", 5.0) or 5.0)
        return pad_graph(g, *self._cap, cutoff)

    def _replay(self, g: AtomicGraph) -> Dict[str, Tensor]:
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

    def _ordinary(self, g: AtomicGraph) -> Dict[str, Tensor]:
        out = self.model(g)
        return {k: v.detach() for k, v in out.items() if torch.is_tensor(v) and v.dim() > 0}

    @staticmethod
    def _timed(fn, g: AtomicGraph):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        out = fn(g)
        b.record()
        torch.cuda.synchronize()
        return out, a.elapsed_time(b)

    def _run_trial(self, g: AtomicGraph) -> None:
        if self.trial <= 0:
            self.replay = True
            return
        rep = min(self._timed(self._replay, g)[1] for _ in range(self.trial))
        ordi = min(self._timed(self._ordinary, g)[1] for _ in range(self.trial))
        self.trial_ms = {"replay": rep, "ordinary": ordi}
        self.replay = rep <= ordi
        if not self.replay:
            self.release()

    # ------------------------------------------------------------------ call
    def __call__(self, g: AtomicGraph) -> Dict[str, Tensor]:
        if g.pos.device.type != "cuda" or self.capturable is False:
            return self._ordinary(g)
        if self.capturable is None:
            out, ms = self._timed(self._ordinary, g)
            self.probes += 1
            if ms <= float(self.max_ms):
                self.capturable = True
            elif self.probes >= PROBES:
                self.capturable = False
            return out
        if not self._fits(g):
            self._capture(g)
            self._run_trial(g)
        if self.replay and self._step is not None:
            return self._replay(g)
        return self._ordinary(g)

    def release(self) -> None:
        if self._step is not None:
            self._step.release()
            self._step = None
