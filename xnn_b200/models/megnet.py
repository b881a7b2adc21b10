"""MEGNet (Chen et al., Chem. Mater. 31, 3564, 2019): graph networks with a global state for
per-structure properties, multi-fidelity with an integer state.

Each block updates bonds, atoms and the state in turn: ``e' = phi_e(v_i + v_j + e + u)``,
``v' = phi_v(v + mean_bonds e' + u)``, ``u' = phi_u(u + mean e' + mean v')`` (``+`` is
concatenation), shifted-softplus dense networks, two dense layers per kind before every block
but the first, a residual around each block. Set2Set readouts of the atoms and bonds and the state
go through a dense network to ``"properties"``. Defaults and parameter names follow the reference
(``src/xnn/gnn/models/megnet.py:67-533``, MatGL's crystal models): 16-wide element embeddings,
100 Gaussians on ``[0, cutoff + 1]`` with exponent 0.5, a 4 A cutoff, two Set2Set steps, a
two-dimensional zero state. Disordered sites take the occupancy-weighted sum of their species'
embeddings.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.blocks import MLP
from ..nn.radial import make_radial_basis
from ..ops.scatter import scatter_sum, segment_softmax
from .base import InteratomicPotential
from .registry import register_model


def _mean(src: Tensor, index: Tensor, count: Tensor) -> Tensor:
    return scatter_sum(src, index, count.shape[0]) / count.clamp(min=1).unsqueeze(-1).to(src.dtype)


class Set2Set(nn.Module):
    """Set2Set readout (Vinyals et al. 2015): an LSTM query, attention over each structure's rows,
    ``q* = [q, r]`` fed back for ``steps`` steps; output ``(B, 2F)``."""

    def __init__(self, n_features: int, steps: int, layers: int = 1):
        super().__init__()
        self.n_features, self.steps, self.layers = int(n_features), int(steps), int(layers)
        self.lstm = nn.LSTM(2 * self.n_features, self.n_features, self.layers)

    def forward(self, x: Tensor, index: Tensor, num_segments: int) -> Tensor:
        h = x.new_zeros((self.layers, num_segments, self.n_features))
        state = (h, h)
        q_star = x.new_zeros((num_segments, 2 * self.n_features))
        for _ in range(self.steps):
            q, state = self.lstm(q_star.unsqueeze(0), state)
            q = q.reshape(num_segments, self.n_features)
            a = segment_softmax((x * q.index_select(0, index)).sum(-1, keepdim=True), index, num_segments)
            q_star = torch.cat([q, scatter_sum(a * x, index, num_segments)], -1)
        return q_star


class _Block(nn.Module):
    def __init__(self, width: int, dense: Optional[Sequence[int]], conv: Sequence[int], activation: str,
                 dropout: float):
        super().__init__()
        conv = [int(c) for c in conv]
        if dense:
            sizes = [width, *[int(d) for d in dense]]
            self.edge_dense = MLP(sizes, activation, activate_last=True)
            self.node_dense = MLP(sizes, activation, activate_last=True)
            self.state_dense = MLP(sizes, activation, activate_last=True)
            inner = sizes[-1]
        else:
            self.edge_dense = self.node_dense = self.state_dense = None
            inner = width
        out = conv[-1]
        self.edge_mlp = MLP([4 * inner, *conv], activation, activate_last=True)
        self.node_mlp = MLP([out + 2 * inner, *conv], activation, activate_last=True)
        self.state_mlp = MLP([2 * out + inner, *conv], activation, activate_last=True)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else None

    def forward(self, e, x, u, dst, src, batch, edge_batch, per_atom, per_bonds, per_atoms):
        e0, x0, u0 = e, x, u
        if self.edge_dense is not None:
            e, x, u = self.edge_dense(e), self.node_dense(x), self.state_dense(u)
        e = self.edge_mlp(torch.cat([x.index_select(0, dst), x.index_select(0, src), e,
                                     u.index_select(0, edge_batch)], -1))
        x = self.node_mlp(torch.cat([x, _mean(e, dst, per_atom), u.index_select(0, batch)], -1))
        u = self.state_mlp(torch.cat([u, _mean(e, edge_batch, per_bonds), _mean(x, batch, per_atoms)], -1))
        if self.dropout is not None:
            e, x, u = self.dropout(e), self.dropout(x), self.dropout(u)
        return e + e0, x + x0, u + u0


@register_model("megnet")
class MEGNet(InteratomicPotential):

    def __init__(self, n_features: int = 16, n_interactions: int = 3, n_rbf: int = 100, cutoff: float = 4.0,
                 rbf_max: Optional[float] = None, gamma: float = 0.5, state_dim: int = 2,
                 n_state_types: Optional[int] = None, state_names: Optional[Sequence[str]] = None,
                 encoder_sizes: Sequence[int] = (64, 32), conv_sizes: Sequence[int] = (64, 64, 32),
                 readout_sizes: Sequence[int] = (32, 16), set2set_steps: int = 2, set2set_layers: int = 1,
                 activation: str = "ssp", dropout: float = 0.0, n_outputs: int = 1, classification: bool = False,
                 n_elements: int = 95, property_scale: float = 1.0, property_shift: float = 0.0):
        super().__init__()
        encoder_sizes = [int(s) for s in encoder_sizes]
        conv_sizes = [int(s) for s in conv_sizes]
        if encoder_sizes[-1] != conv_sizes[-1]:
            raise ValueError("the residual of the first block needs the last encoder size to equal the last "
                             f"conv size ({encoder_sizes[-1]} != {conv_sizes[-1]})")
        if n_state_types is not None and state_names is not None and len(state_names) != n_state_types:
            raise ValueError(f"got {len(state_names)} state names for {n_state_types} state types")
        self.cutoff = float(cutoff)
        self.n_state_types = None if n_state_types is None else int(n_state_types)
        self.state_dim = int(state_dim)
        self.state_names = None if state_names is None else [str(s) for s in state_names]
        self.n_outputs = int(n_outputs)
        self.classification = bool(classification)
        self.rbf = make_radial_basis("gaussian", int(n_rbf), self.cutoff + 1.0 if rbf_max is None else float(rbf_max),
                                     gamma=float(gamma))
        self.node_embedding = nn.Embedding(int(n_elements), int(n_features))
        self.state_embedding = (nn.Embedding(self.n_state_types, self.state_dim)
                                if self.n_state_types is not None else None)
        self.edge_encoder = MLP([int(n_rbf), *encoder_sizes], activation, activate_last=True)
        self.node_encoder = MLP([int(n_features), *encoder_sizes], activation, activate_last=True)
        self.state_encoder = MLP([self.state_dim, *encoder_sizes], activation, activate_last=True)
        width = conv_sizes[-1]
        self.blocks = nn.ModuleList(_Block(width, None if k == 0 else encoder_sizes, conv_sizes, activation,
                                           float(dropout)) for k in range(int(n_interactions)))
        self.node_set2set = Set2Set(width, set2set_steps, set2set_layers)
        self.edge_set2set = Set2Set(width, set2set_steps, set2set_layers)
        self.dropout = nn.Dropout(float(dropout)) if dropout > 0 else None
        self.readout = MLP([5 * width, *[int(s) for s in readout_sizes], self.n_outputs], activation)
        self.register_buffer("property_scale", torch.tensor(float(property_scale)))
        self.register_buffer("property_shift", torch.tensor(float(property_shift)))

    def state_label(self, name: str) -> int:
        if self.state_names is None or name not in self.state_names:
            raise KeyError(f"unknown state {name!r}; known: {self.state_names}")
        return self.state_names.index(name)

    def set_property_scale_shift(self, scale: float, shift: float) -> None:
        self.property_scale.fill_(float(scale))
        self.property_shift.fill_(float(shift))

    def _sites(self, data: AtomicGraph) -> Tensor:
        if data.site_species is None:
            return self.node_embedding(data.atomic_numbers)
        w = data.site_occupancy.to(self.node_embedding.weight.dtype)
        return (self.node_embedding(data.site_species) * w.unsqueeze(-1)).sum(1)

    def _state(self, data: AtomicGraph, dtype) -> Tensor:
        b, dev = data.num_graphs, data.pos.device
        if self.state_embedding is not None:
            labels = torch.zeros(b, dtype=torch.long, device=dev) if data.state is None else data.state.reshape(b).long()
            return self.state_embedding(labels)
        if data.state is None:
            return torch.zeros((b, self.state_dim), dtype=dtype, device=dev)
        return data.state.reshape(b, self.state_dim).to(dtype)

    def forward(self, data: AtomicGraph) -> dict:
        src, dst = data.edge_index[0], data.edge_index[1]
        b, n, batch = data.num_graphs, data.num_nodes, data.batch
        edge_batch = batch.index_select(0, dst)
        dist = data.edge_vectors().norm(dim=-1)
        per_atom, per_bonds = torch.bincount(dst, minlength=n), torch.bincount(edge_batch, minlength=b)
        x, u = self._sites(data), self._state(data, dist.dtype)
        e, x, u = self.edge_encoder(self.rbf(dist)), self.node_encoder(x), self.state_encoder(u)
        for block in self.blocks:
            e, x, u = block(e, x, u, dst, src, batch, edge_batch, per_atom, per_bonds, data.n_atoms)
        features = torch.cat([self.node_set2set(x, batch, b), self.edge_set2set(e, edge_batch, b), u], -1)
        y = self.readout(features if self.dropout is None else self.dropout(features))
        if self.classification:
            y = torch.sigmoid(y)
        y = self.property_scale * y + self.property_shift
        return {"properties": y.squeeze(-1) if self.n_outputs == 1 else y, "structure_features": features}

    @classmethod
    def from_config(cls, cfg) -> "MEGNet":
        e = dict(cfg.extra or {})
        keys = ("rbf_max", "gamma", "state_dim", "n_state_types", "state_names", "encoder_sizes", "conv_sizes",
                "readout_sizes", "set2set_steps", "set2set_layers", "activation", "dropout", "n_outputs",
                "classification", "n_elements", "property_scale", "property_shift")
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf, cutoff=cfg.cutoff,
                   **{k: e[k] for k in keys if k in e})
