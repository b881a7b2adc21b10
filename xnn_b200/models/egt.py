"""Edge-augmented graph transformer (EGT; Hussain et al., KDD 2022) over two-dimensional molecular
graphs, the trunk of graph-parameterised force fields (ByteFF): integer atom and bond features are
embedded and averaged over topologically equivalent atoms / bonds, then pre-norm attention layers
update node and edge channels together (edge-biased, edge-gated attention; the logits feed back into
the edges), with jumping-knowledge output and bond features symmetrised over both directions.

Feature tables, layer structure and parameter names follow the reference
(``src/xnn/gnn/models/egt.py``) so state dicts transplant.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from ..nn.blocks import MLP, make_activation

N_ELEMENTS, MAX_DEGREE, MAX_FORMAL_CHARGE, MAX_RING = 86, 6, 2, 8
N_BOND_RING, N_BOND_ORDER = 2, 4


def class_mean(x: Tensor, cls: Tensor) -> Tensor:
    """Every row replaced by the average of the rows that share its class label."""
    n = x.shape[0]
    sums = x.new_zeros((n,) + tuple(x.shape[1:])).index_add_(0, cls, x)
    sizes = torch.bincount(cls, minlength=n).clamp_min(1).to(x.dtype)
    return (sums / sizes.view(-1, *([1] * (x.dim() - 1)))).index_select(0, cls)


def _segment_softmax(logits: Tensor, seg: Tensor, n: int) -> Tensor:
    """Softmax of ``logits (E, H)`` within each group of rows sharing ``seg`` (max-shifted)."""
    top = logits.new_full((n, logits.shape[1]), float("-inf"))
    top = top.index_reduce_(0, seg, logits.detach(), "amax")
    ex = torch.exp(logits - top.index_select(0, seg))
    den = ex.new_zeros((n, ex.shape[1])).index_add_(0, seg, ex)
    return ex / den.index_select(0, seg)


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
        # column c of the integer feature table goes through table c; the formal charge is shifted
        # into the table's range and clipped
        cols = node_features.unbind(-1)
        shifted = (cols[2] + MAX_FORMAL_CHARGE).clamp(0, 2 * MAX_FORMAL_CHARGE)
        atom_tables = (self.element, self.degree, self.formal_charge, self.ring_degree, self.min_ring)
        atom_cols = (cols[0], cols[1], shifted, cols[3], cols[4])
        atoms = torch.cat([tab(c) for tab, c in zip(atom_tables, atom_cols)], dim=-1)
        bcols = edge_features.unbind(-1)
        bonds = torch.cat([self.bond_ring(bcols[0]), self.bond_order(bcols[1])], dim=-1)
        return class_mean(self.node_mlp(atoms), atom_class), class_mean(self.edge_mlp(bonds), edge_class)


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

    def _qkv(self, h: Tensor):
        """Query, key and value heads from one matrix product over the stacked projections."""
        w = torch.cat([self.query.weight, self.key.weight, self.value.weight], 0)
        b = torch.cat([self.query.bias, self.key.bias, self.value.bias], 0)
        return F.linear(h, w, b).view(h.shape[0], 3, self.heads, self.head_dim).unbind(1)

    def forward(self, x: Tensor, e: Tensor, src: Tensor, dst: Tensor):
        n = x.shape[0]
        q, k, v = self._qkv(self.norm1(x))
        ge = self.edge_norm1(e)
        # per edge and head: scaled dot product of the receiver's query with the sender's key,
        # biased by the edge channels; the same logits later feed back into the edges
        logits = torch.einsum("ehc,ehc->eh", q[dst], k[src]) * self.head_dim ** -0.5 + self.edge_bias(ge)
        att = _segment_softmax(logits, dst, n) * torch.sigmoid(self.gate(ge))
        if self.scale_by_degree:
            att = att * torch.bincount(dst, minlength=n).to(att.dtype)[dst, None]
        agg = x.new_zeros((n, self.heads, self.head_dim)).index_add_(0, dst, v[src] * att[..., None])
        x = x + self.proj(agg.flatten(1))
        x = x + self.ffn(self.norm2(x))
        e = e + self.edge_proj(logits)
        e = e + self.edge_ffn(self.edge_norm2(e))
        return x, e


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
        src, dst = edge_index.unbind(0)
        history = []
        n_layers = len(self.layers)
        for depth, layer in enumerate(self.layers, start=1):
            x, e = layer(x, e, src, dst)
            # the activation follows every layer but the last, and the last too when an output
            # head (jumping knowledge) comes after it
            if depth < n_layers or self.jumping_knowledge is not None:
                x = self.act(x)
            history.append(x)
        if self.out is not None:
            x = self.out(torch.cat(history, -1) if self.jumping_knowledge == "cat" else x)
        e = self.edge_out(e)
        # both directions of a bond (consecutive rows) carry the average of the two
        pairs = e.view(-1, 2, e.shape[-1])
        e = pairs.mean(1, keepdim=True).expand_as(pairs).reshape(e.shape)
        return x, e
