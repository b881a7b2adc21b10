"""CGCNN (Xie & Grossman, PRL 120, 145301, 2018): crystal graph convolutions for per-structure
properties.

Atoms start from a fixed element feature table mapped by a dense layer; bonds (the ``k`` nearest
neighbours within the cutoff) carry Gaussians of their length; each convolution updates
``v_i <- g(v_i + BN(sum_j sigmoid(BN1(z W_f)) * g(BN1(z W_s))))`` with ``z = [v_i, v_j, u_ij]`` and
``g`` the softplus; the mean over a structure goes through softplus dense layers to the output
(``"properties"``, or a two-class probability). Options, defaults and parameter names follow the
reference (``src/xnn/gnn/models/cgcnn.py:92-495``): 12 neighbours within 8 A, 41 Gaussians
``exp(-(r - mu)^2 / 0.2^2)``, 64 features, 3 convolutions, one hidden layer of 128.

The authors' 92-column element table is not bundled (it is downloaded by the reference); with
``atom_features="cgcnn"`` the table comes from a checkpoint's state dict, or from the JSON file
named by ``$XNN_B200_CGCNN_TABLE`` (the authors' ``atom_init.json`` format), on first use.
"""
from __future__ import annotations

import json
import os
from pathlib import Path
from typing import Optional, Sequence

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..data.neighborlist import nearest_edges
from ..nn.blocks import exact_softplus
from ..nn.radial import GaussianRBF
from ..ops.scatter import scatter_sum
from .base import InteratomicPotential
from .registry import register_model

TABLE_SHAPE = (101, 92)


def read_atom_features(spec, n_elements: int = TABLE_SHAPE[0]) -> Tensor:
    """An element table (row ``Z`` for atomic number ``Z``) from ``"onehot"``, a JSON file in the
    ``atom_init.json`` format, a mapping ``Z -> vector`` or an array."""
    if isinstance(spec, str) and spec == "onehot":
        return torch.eye(int(n_elements), dtype=torch.float64)
    if isinstance(spec, (str, Path)):
        with open(spec) as f:
            spec = json.load(f)
    if isinstance(spec, dict):
        rows = {int(z): torch.as_tensor(v, dtype=torch.float64).reshape(-1) for z, v in spec.items()}
        widths = {v.numel() for v in rows.values()}
        if len(widths) != 1:
            raise ValueError(f"element feature vectors of different lengths: {sorted(widths)}")
        table = torch.zeros(max(rows) + 1, widths.pop(), dtype=torch.float64)
        for z, v in rows.items():
            table[z] = v
        return table
    table = torch.as_tensor(spec, dtype=torch.float64)
    if table.dim() != 2:
        raise ValueError(f"an element feature table has two dimensions, got {tuple(table.shape)}")
    return table


class ConvLayer(nn.Module):
    def __init__(self, n_features: int, n_rbf: int, normalization: Optional[str] = "batch",
                 residual_activation: bool = True):
        super().__init__()
        f = int(n_features)
        self.fc_full = nn.Linear(2 * f + int(n_rbf), 2 * f)
        self.bn1 = nn.BatchNorm1d(2 * f) if normalization == "batch" else None
        self.bn2 = nn.BatchNorm1d(f) if normalization == "batch" else None
        self.residual_activation = bool(residual_activation)

    def forward(self, x: Tensor, u: Tensor, src: Tensor, dst: Tensor) -> Tensor:
        n, f = x.shape
        # the layer split by input: the receiver's and sender's parts once per atom, the bond part per edge
        w = self.fc_full.weight
        atoms = torch.nn.functional.linear(x, torch.cat([w[:, :f], w[:, f:2 * f]]))
        h = (torch.nn.functional.linear(u, w[:, 2 * f:], self.fc_full.bias)
             + atoms[:, :2 * f].index_select(0, dst) + atoms[:, 2 * f:].index_select(0, src))
        if self.bn1 is not None:
            h = self.bn1(h)
        gate, core = h.chunk(2, dim=-1)
        s = scatter_sum(torch.sigmoid(gate) * exact_softplus(core), dst, n)
        if self.bn2 is not None:
            s = self.bn2(s)
        out = x + s
        return exact_softplus(out) if self.residual_activation else out


@register_model("cgcnn")
class CGCNN(InteratomicPotential):

    def __init__(self, n_features: int = 64, n_interactions: int = 3, n_rbf: int = 41, cutoff: float = 8.0,
                 max_neighbors: Optional[int] = 12, rbf_start: float = 0.0, rbf_max: Optional[float] = None,
                 gamma: Optional[float] = None, readout_sizes: Sequence[int] = (128,),
                 normalization: Optional[str] = "batch", residual_activation: bool = True, n_outputs: int = 1,
                 classification: bool = False, dropout: Optional[float] = None, atom_features="cgcnn",
                 n_elements: int = TABLE_SHAPE[0], property_scale: float = 1.0, property_shift: float = 0.0):
        super().__init__()
        readout_sizes = [int(s) for s in readout_sizes]
        if not readout_sizes:
            raise ValueError("CGCNN needs at least one hidden layer after the pooling")
        if normalization not in ("batch", None):
            raise ValueError(f"normalization must be 'batch' or None, got {normalization!r}")
        self.cutoff = float(cutoff)
        self.max_neighbors = None if max_neighbors is None else int(max_neighbors)
        self.classification = bool(classification)
        self.n_outputs = 2 if self.classification else int(n_outputs)
        rbf_max = self.cutoff if rbf_max is None else float(rbf_max)
        n_rbf = int(n_rbf)
        if gamma is None:
            gamma = 1.0 / ((rbf_max - float(rbf_start)) / (n_rbf - 1)) ** 2 if n_rbf > 1 else 1.0
        self.rbf = GaussianRBF(n_rbf, rbf_max, start=float(rbf_start), gamma=float(gamma))
        self._table_pending = isinstance(atom_features, str) and atom_features == "cgcnn"
        table = (torch.zeros(TABLE_SHAPE, dtype=torch.float64) if self._table_pending
                 else read_atom_features(atom_features, n_elements))
        self.register_buffer("atom_features", table.to(torch.get_default_dtype()))
        f = int(n_features)
        self.embedding = nn.Linear(table.shape[1], f)
        self.convs = nn.ModuleList(ConvLayer(f, n_rbf, normalization, residual_activation)
                                   for _ in range(int(n_interactions)))
        self.conv_to_fc = nn.Linear(f, readout_sizes[0])
        self.fcs = nn.ModuleList(nn.Linear(a, b) for a, b in zip(readout_sizes[:-1], readout_sizes[1:]))
        self.fc_out = nn.Linear(readout_sizes[-1], self.n_outputs)
        p = (0.5 if self.classification else 0.0) if dropout is None else float(dropout)
        self.dropout = nn.Dropout(p) if p > 0 else None
        self.register_buffer("property_scale", torch.tensor(float(property_scale)))
        self.register_buffer("property_shift", torch.tensor(float(property_shift)))

    def _ensure_table(self) -> None:
        if not self._table_pending:
            return
        path = os.environ.get("XNN_B200_CGCNN_TABLE")
        if not path:
            raise RuntimeError("CGCNN's element table is not loaded: load a checkpoint that holds it, pass "
                               "atom_features (a table, a mapping or 'onehot'), or name the authors' "
                               "atom_init.json in $XNN_B200_CGCNN_TABLE")
        with torch.no_grad():
            t = read_atom_features(path)
            self.atom_features.zero_()
            self.atom_features[:t.shape[0]].copy_(t[:TABLE_SHAPE[0]].to(self.atom_features))
        self._table_pending = False

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        if prefix + "atom_features" in state_dict:
            self._table_pending = False
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def set_property_scale_shift(self, scale: float, shift: float) -> None:
        self.property_scale.fill_(float(scale))
        self.property_shift.fill_(float(shift))

    def forward(self, data: AtomicGraph) -> dict:
        self._ensure_table()
        src, dst = data.edge_index[0], data.edge_index[1]
        n, b = data.num_nodes, data.num_graphs
        dist = data.edge_vectors().norm(dim=-1)
        if self.max_neighbors is not None and dst.numel():
            keep = torch.nonzero(nearest_edges(data.edge_index, dist.detach(), self.max_neighbors, n)).flatten()
            src, dst, dist = src.index_select(0, keep), dst.index_select(0, keep), dist.index_select(0, keep)
        u = self.rbf(dist)
        x = self.embedding(self.atom_features.index_select(0, data.atomic_numbers))
        for conv in self.convs:
            x = conv(x, u, src, dst)
        pooled = scatter_sum(x, data.batch, b) / data.n_atoms.clamp(min=1).unsqueeze(-1).to(x.dtype)
        h = exact_softplus(self.conv_to_fc(exact_softplus(pooled)))
        if self.dropout is not None:
            h = self.dropout(h)
        for fc in self.fcs:
            h = exact_softplus(fc(h))
        y = self.fc_out(h)
        out = {"structure_features": pooled}
        if self.classification:
            log_p = torch.log_softmax(y, dim=-1)
            out["log_probabilities"] = log_p
            out["properties"] = log_p[:, 1].exp()
            return out
        y = torch.addcmul(self.property_shift, self.property_scale, y)
        out["properties"] = y.squeeze(-1) if self.n_outputs == 1 else y
        return out

    @classmethod
    def from_config(cls, cfg) -> "CGCNN":
        e = dict(cfg.extra or {})
        keys = ("max_neighbors", "rbf_start", "rbf_max", "gamma", "readout_sizes", "normalization",
                "residual_activation", "n_outputs", "classification", "dropout", "atom_features", "n_elements",
                "property_scale", "property_shift")
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf, cutoff=cfg.cutoff,
                   **{k: e[k] for k in keys if k in e})
