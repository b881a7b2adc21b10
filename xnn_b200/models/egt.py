"""Edge-augmented graph transformer (EGT; Hussain et al., KDD 2022) over two-dimensional molecular
graphs, the trunk of graph-parameterised force fields (ByteFF): integer atom and bond features are
embedded and averaged over topologically equivalent atoms / bonds, then pre-norm attention layers
update node and edge channels together (edge-biased, edge-gated attention; the logits feed back into
the edges), with jumping-knowledge output and bond features symmetrised over both directions.

Feature tables, layer structure and parameter names follow the reference
(``src/xnn/gnn/models/egt.py``) so state dicts transplant.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor, nn

from ..nn.blocks import MLP, make_activation
from ..ops.scatter import scatter_sum

N_ELEMENTS, MAX_DEGREE, MAX_FORMAL_CHARGE, MAX_RING = 86, 6, 2, 8
N_BOND_RING, N_BOND_ORDER = 2, 4


def class_mean(x: Tensor, cls: Tensor) -> Tensor:
    """Each row replaced by the mean of the rows of its class."""
    n = x.shape[0]
    total = scatter_sum(x, cls, n)
    count = scatter_sum(torch.ones_like(cls, dtype=x.dtype), cls, n)
    return (total / count.clamp(min=1.0).unsqueeze(-1)).index_select(0, cls)


def _mlp(n_in: int, hidden: int, n_out: int, layers: int, activation, activate_last: bool = False) -> MLP:
    return MLP([n_in] + [hidden] * (layers - 1) + [n_out], activation, activate_last=activate_last)


class GraphEmbedding(nn.Module):
    """Atom features ``(element, degree, formal charge, ring degree, smallest ring)`` and bond
    features ``(in ring, order)`` embedded, passed through MLPs and averaged per equivalence class."""

    def __init__(self, atom_dim: int = 32, feature_dim: int = 8, node_mlp=(64, 256, 2), edge_mlp=(64, 256, 2),
                 activation: str = "gelu"):
        super().__init__()
        self.element = nn.Embedding(N_ELEMENTS, atom_dim)
        self.degree = nn.Embedding(MAX_DEGREE + 1, feature_dim)
        self.formal_charge = nn.Embedding(2 * MAX_FORMAL_CHARGE + 1, feature_dim)
        self.ring_degree = nn.Embedding(MAX_DEGREE + 1, feature_dim)
        self.min_ring = nn.Embedding(MAX_RING + 1, feature_dim)
        self.bond_ring = nn.Embedding(N_BOND_RING, feature_dim)
        self.bond_order = nn.Embedding(N_BOND_ORDER, feature_dim)
        self.node_mlp = _mlp(atom_dim + 4 * feature_dim, node_mlp[0], node_mlp[1], node_mlp[2], activation, True)
        self.edge_mlp = _mlp(2 * feature_dim, edge_mlp[0], edge_mlp[1], edge_mlp[2], activation, True)
        self.node_dim, self.edge_dim = int(node_mlp[1]), int(edge_mlp[1])

    def forward(self, node_features: Tensor, edge_features: Tensor, atom_class: Tensor, edge_class: Tensor):
        f = node_features
        charge = torch.clamp(f[:, 2] + MAX_FORMAL_CHARGE, 0, 2 * MAX_FORMAL_CHARGE)
        x = torch.cat([self.element(f[:, 0]), self.degree(f[:, 1]), self.formal_charge(charge),
                       self.ring_degree(f[:, 3]), self.min_ring(f[:, 4])], -1)
        e = torch.cat([self.bond_ring(edge_features[:, 0]), self.bond_order(edge_features[:, 1])], -1)
        return class_mean(self.node_mlp(x), atom_class), class_mean(self.edge_mlp(e), edge_class)


class EGTLayer(nn.Module):
    """Multi-head attention along the directed bonds with edge bias and sigmoid edge gates; the
    logits update the edge channels; pre-norm residual feed-forward blocks on both."""

    def __init__(self, dim: int, heads: int = 16, head_dim: int = 16, ffn=(256, 2), activation: str = "gelu",
                 scale_by_degree: bool = False):
        super().__init__()
        self.heads, self.head_dim, self.scale_by_degree = int(heads), int(head_dim), bool(scale_by_degree)
        width = self.heads * self.head_dim
        self.query, self.key, self.value = (nn.Linear(dim, width) for _ in range(3))
        self.proj = nn.Linear(width, dim)
        self.norm1, self.norm2 = nn.LayerNorm(dim), nn.LayerNorm(dim)
        self.gate = nn.Linear(dim, self.heads)
        self.edge_bias = nn.Linear(dim, self.heads)
        self.edge_proj = nn.Linear(self.heads, dim)
        self.edge_norm1, self.edge_norm2 = nn.LayerNorm(dim), nn.LayerNorm(dim)
        self.ffn = _mlp(dim, ffn[0], dim, ffn[1], activation)
        self.edge_ffn = _mlp(dim, ffn[0], dim, ffn[1], activation)

    def forward(self, x: Tensor, e: Tensor, src: Tensor, dst: Tensor):
        n, H, C = x.shape[0], self.heads, self.head_dim
        h = self.norm1(x)
        q, k, v = self.query(h).view(n, H, C), self.key(h).view(n, H, C), self.value(h).view(n, H, C)
        g = self.edge_norm1(e)
        gate = torch.sigmoid(self.gate(g))
        logits = (q.index_select(0, dst) * k.index_select(0, src)).sum(-1) / math.sqrt(C) + self.edge_bias(g)
        peak = torch.full((n, H), float("-inf"), dtype=logits.dtype, device=logits.device)
        peak = peak.scatter_reduce(0, dst.unsqueeze(-1).expand(-1, H), logits.detach(), "amax")
        w = torch.exp(logits - peak.index_select(0, dst))
        w = w / scatter_sum(w, dst, n).index_select(0, dst)
        if self.scale_by_degree:
            w = w * scatter_sum(torch.ones_like(dst, dtype=w.dtype), dst, n).index_select(0, dst).unsqueeze(-1)
        msg = v.index_select(0, src) * (gate * w).unsqueeze(-1)
        x = self.proj(scatter_sum(msg, dst, n).reshape(n, H * C)) + x
        x = self.ffn(self.norm2(x)) + x
        e = e + self.edge_proj(logits)
        return x, self.edge_ffn(self.edge_norm2(e)) + e


class MolecularGraphTransformer(nn.Module):
    """Node features ``(N, node_dim)`` and per-directed-bond features ``(2M, edge_dim)`` (both
    directions of a bond equal) of molecular graphs whose bonds are listed as consecutive direction
    pairs."""

    def __init__(self, atom_dim: int = 32, feature_dim: int = 8, node_mlp=(64, 256, 2), edge_mlp=(64, 256, 2),
                 hidden: int = 256, layers: int = 4, heads: int = 16, head_dim: int = 16, ffn=(256, 2),
                 out_dim: int = 256, jumping_knowledge: Optional[str] = "cat", activation: str = "gelu",
                 scale_by_degree: bool = False):
        super().__init__()
        if jumping_knowledge not in ("cat", "last", None):
            raise ValueError(f"jumping_knowledge must be 'cat', 'last' or None, got {jumping_knowledge!r}")
        self.embedding = GraphEmbedding(atom_dim, feature_dim, node_mlp, edge_mlp, activation)
        node_in, edge_in = self.embedding.node_dim, self.embedding.edge_dim
        if hidden != node_in:
            raise ValueError(f"the attention width must equal the node embedding width ({hidden} != {node_in})")
        if jumping_knowledge is None and out_dim != hidden:
            raise ValueError("without jumping knowledge out_dim must equal hidden")
        self.jumping_knowledge = jumping_knowledge
        self.edge_in = nn.Linear(edge_in, hidden)
        self.layers = nn.ModuleList(EGTLayer(hidden, heads, head_dim, ffn, activation, scale_by_degree)
                                    for _ in range(int(layers)))
        self.act = make_activation(activation)
        self.edge_out = nn.Linear(hidden, edge_in)
        self.out = None
        if jumping_knowledge is not None:
            self.out = nn.Linear(hidden * int(layers) if jumping_knowledge == "cat" else hidden, out_dim)
        self.node_dim, self.edge_dim = int(out_dim), int(edge_in)

    def forward(self, node_features: Tensor, edge_features: Tensor, edge_index: Tensor, atom_class: Tensor,
                edge_class: Tensor):
        x, e = self.embedding(node_features, edge_features, atom_class, edge_class)
        e = self.edge_in(e)
        src, dst = edge_index[0], edge_index[1]
        outs, last = [], len(self.layers) - 1
        for i, layer in enumerate(self.layers):
            x, e = layer(x, e, src, dst)
            if i < last or self.jumping_knowledge is not None:
                x = self.act(x)
            outs.append(x)
        if self.jumping_knowledge == "cat":
            x = self.out(torch.cat(outs, -1))
        elif self.jumping_knowledge == "last":
            x = self.out(x)
        e = self.edge_out(e)
        m = e.shape[0] // 2
        e = (0.5 * (e[0::2] + e[1::2])).unsqueeze(1).expand(m, 2, e.shape[1]).reshape(2 * m, e.shape[1])
        return x, e
