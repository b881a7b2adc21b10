"""The equivariant transformer of TorchMD-Net (Thoelke & De Fabritiis, ICLR 2022).

Scalar features ``x`` and vector features ``v (N, 3, F)``; a neighbour embedding; per layer a
multi-head attention over the graph's edges plus self loops with distance-filtered keys and
values (``distance_influence``), messages ``v_j * a + direction * b`` for the vectors, the
update ``dx = (v1 . v2) o2 + o3``, ``dv = v3 o1 + sum``; a final LayerNorm and two gated
equivariant blocks to the atomic energy. Options, initialisation and parameter names follow the
reference (``src/xnn/trfnn/models/et.py``) so that weights transplant.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.blocks import GatedEquivariantBlock, make_activation
from ..nn.cutoff import CosineCutoff
from ..nn.radial import make_radial_basis
from ..ops.scatter import scatter_sum
from .base import InteratomicPotential
from .registry import register_model

_INFLUENCES = ("both", "keys", "values", "none")


def _xavier_zero_bias_(module: nn.Module) -> None:
    for m in module.modules():
        if isinstance(m, nn.Linear):
            nn.init.xavier_uniform_(m.weight)
            if m.bias is not None:
                nn.init.zeros_(m.bias)


class TransformerPotential(InteratomicPotential):
    """Energy scale / shift buffers and per-element reference energies of the transformer models."""
    head_modules = ("readout", "energy_scale", "energy_shift", "atom_ref")

    def _init_energy_terms(self, n_elements: int, energy_scale: float, energy_shift: float, species=None,
                           atomic_energies=None) -> None:
        self.register_buffer("energy_scale", torch.tensor(float(energy_scale)))
        self.register_buffer("energy_shift", torch.tensor(float(energy_shift)))
        self.atom_ref = nn.Embedding(n_elements, 1)
        nn.init.zeros_(self.atom_ref.weight)
        if atomic_energies is not None:
            if species is None:
                raise ValueError("species is required to map atomic_energies")
            self.set_atomic_energies(species, atomic_energies)

    def set_energy_scale_shift(self, scale: float, shift: float) -> None:
        with torch.no_grad():
            self.energy_scale.fill_(float(scale))
            self.energy_shift.fill_(float(shift))

    def set_atomic_energies(self, species, values) -> None:
        with torch.no_grad():
            self.atom_ref.weight[torch.tensor(list(species)), 0] = torch.as_tensor(values,
                                                                                   dtype=self.atom_ref.weight.dtype)


class _NeighborEmbedding(nn.Module):
    def __init__(self, n: int, n_rbf: int, n_elements: int):
        super().__init__()
        self.embedding = nn.Embedding(n_elements, n)
        self.distance_proj = nn.Linear(n_rbf, n)
        self.combine = nn.Linear(2 * n, n)
        _xavier_zero_bias_(self)

    def forward(self, z, x, src, dst, envelope, rbf):
        w = self.distance_proj(rbf) * envelope.unsqueeze(-1)
        nb = scatter_sum(w * self.embedding(z).index_select(0, src), dst, x.shape[0])
        return self.combine(torch.cat([x, nb], -1))


class _AttentionLayer(nn.Module):
    def __init__(self, n: int, n_rbf: int, heads: int, activation: str, attn_activation: str, influence: str,
                 vector_cutoff: bool):
        super().__init__()
        self.n_features, self.num_heads, self.head_dim = n, heads, n // heads
        self.vector_cutoff = vector_cutoff
        self.layernorm = nn.LayerNorm(n)
        self.act, self.attn_act = make_activation(activation), make_activation(attn_activation)
        self.q_proj, self.k_proj = nn.Linear(n, n), nn.Linear(n, n)
        self.v_proj, self.o_proj = nn.Linear(n, 3 * n), nn.Linear(n, 3 * n)
        self.vec_proj = nn.Linear(n, 3 * n, bias=False)
        self.dk_proj = nn.Linear(n_rbf, n) if influence in ("keys", "both") else None
        self.dv_proj = nn.Linear(n_rbf, 3 * n) if influence in ("values", "both") else None
        _xavier_zero_bias_(self)

    def forward(self, x, vec, src, dst, envelope, rbf, direction):
        n, F, H, d = x.shape[0], self.n_features, self.num_heads, self.head_dim
        x = self.layernorm(x)
        q, k = self.q_proj(x).reshape(n, H, d), self.k_proj(x).reshape(n, H, d)
        v = self.v_proj(x).reshape(n, H, 3 * d)
        vec1, vec2, vec3 = torch.split(self.vec_proj(vec), F, dim=-1)
        logits = q.index_select(0, dst) * k.index_select(0, src)
        if self.dk_proj is not None:
            logits = logits * self.act(self.dk_proj(rbf)).reshape(-1, H, d)
        attn = self.attn_act(logits.sum(-1))
        values = v.index_select(0, src)
        if self.vector_cutoff:
            values = values * envelope[:, None, None]
        else:
            attn = attn * envelope[:, None]
        if self.dv_proj is not None:
            values = values * self.act(self.dv_proj(rbf)).reshape(-1, H, 3 * d)
        v0, v1, v2 = torch.split(values, d, dim=-1)
        dx = scatter_sum(v0 * attn.unsqueeze(-1), dst, n)
        msg_vec = vec.reshape(n, 3, H, d).index_select(0, src) * v1.unsqueeze(1) + \
            v2.unsqueeze(1) * direction[:, :, None, None]
        dvec = scatter_sum(msg_vec, dst, n)
        o1, o2, o3 = torch.split(self.o_proj(dx.reshape(n, F)), F, dim=-1)
        return (vec1 * vec2).sum(1) * o2 + o3, vec3 * o1.unsqueeze(1) + dvec.reshape(n, 3, F), attn


class _EquivariantScalar(nn.Module):
    def __init__(self, n: int, activation: str):
        super().__init__()
        h = n // 2
        self.blocks = nn.ModuleList([
            GatedEquivariantBlock(n, n, h, h, n_hidden=n, scalar_activation=True, n_norm=n, activation=activation),
            GatedEquivariantBlock(h, h, 1, 1, n_hidden=h, scalar_activation=False, n_norm=h, activation=activation)])
        _xavier_zero_bias_(self)

    def forward(self, x, vec):
        for blk in self.blocks:
            x, vec = blk(x, vec)
        return x.squeeze(-1)


@register_model("et")
class EquivariantTransformer(TransformerPotential):
    def __init__(self, n_features: int = 128, n_interactions: int = 6, n_rbf: int = 32, cutoff: float = 5.0,
                 num_heads: int = 8, radial_basis: str = "expnorm", trainable_rbf: bool = False,
                 activation: str = "silu", attn_activation: str = "silu", neighbor_embedding: bool = True,
                 distance_influence: str = "both", vector_cutoff: bool = True, n_elements: int = 100,
                 energy_shift: float = 0.0, energy_scale: float = 1.0, species=None, atomic_energies=None):
        super().__init__()
        if n_features % num_heads:
            raise ValueError(f"n_features ({n_features}) must be divisible by num_heads ({num_heads})")
        if distance_influence not in _INFLUENCES:
            raise ValueError(f"distance_influence must be one of {_INFLUENCES}, got {distance_influence!r}")
        self.cutoff = float(cutoff)
        if species is not None:
            self.species = [int(z) for z in species]
        self.n_features = self.node_feature_dim = n_features
        self.n_interactions, self.num_heads = n_interactions, num_heads
        self.distance_influence, self.vector_cutoff = distance_influence, vector_cutoff
        self.embedding = nn.Embedding(n_elements, n_features)
        self.rbf = make_radial_basis(radial_basis, n_rbf, cutoff, trainable_rbf)
        self.cutoff_fn = CosineCutoff(cutoff)
        self.neighbor_embedding = _NeighborEmbedding(n_features, n_rbf, n_elements) if neighbor_embedding else None
        self.layers = nn.ModuleList([_AttentionLayer(n_features, n_rbf, num_heads, activation, attn_activation,
                                                     distance_influence, vector_cutoff) for _ in range(n_interactions)])
        self.out_norm = nn.LayerNorm(n_features)
        self.readout = _EquivariantScalar(n_features, activation)
        self._init_energy_terms(n_elements, energy_scale, energy_shift, species, atomic_energies)

    def receptive_field(self) -> float:
        return max(1, self.n_interactions) * self.cutoff

    def _pairs(self, edge_index: Tensor, edge_vec: Tensor, n: int):
        r = torch.linalg.norm(edge_vec, dim=-1)
        direction = -edge_vec / r.clamp(min=1e-12).unsqueeze(-1)
        loops = torch.arange(n, dtype=edge_index.dtype, device=edge_index.device)
        src, dst = torch.cat([edge_index[0], loops]), torch.cat([edge_index[1], loops])
        r = torch.cat([r, r.new_zeros(n)])
        direction = torch.cat([direction, direction.new_zeros(n, 3)])
        return src, dst, self.cutoff_fn(r), self.rbf(r), direction

    def representation(self, z: Tensor, edge_index: Tensor, edge_vec: Tensor, attention: Optional[List] = None):
        src, dst, env, rbf, direction = self._pairs(edge_index, edge_vec, z.shape[0])
        x = self.embedding(z)
        e = edge_index.shape[1]
        if self.neighbor_embedding is not None:
            x = self.neighbor_embedding(z, x, edge_index[0], edge_index[1], env[:e], rbf[:e])
        vec = x.new_zeros(x.shape[0], 3, x.shape[1])
        for layer in self.layers:
            dx, dvec, attn = layer(x, vec, src, dst, env, rbf, direction)
            x, vec = x + dx, vec + dvec
            if attention is not None:
                attention.append(attn[:e])
        return self.out_norm(x), vec

    def attention_weights(self, data: AtomicGraph) -> List[Tensor]:
        out: List[Tensor] = []
        self.representation(data.atomic_numbers, data.edge_index, data.edge_vectors(), out)
        return out

    def _energy(self, x, vec, z):
        return self.energy_scale * self.readout(x, vec) + self.energy_shift + self.atom_ref(z).squeeze(-1)

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        x, vec = self.representation(atomic_numbers, edge_index, edge_vec)
        return x, self._energy(x, vec, atomic_numbers)

    def node_energy(self, atomic_numbers, edge_index, edge_vec):
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> dict:
        x, vec = self.representation(data.atomic_numbers, data.edge_index, data.edge_vectors())
        e = self._energy(x, vec, data.atomic_numbers)
        return {"node_energy": e, "energy": self.aggregate_energy(e, data), "node_features": x, "node_vectors": vec}

    @classmethod
    def from_config(cls, cfg) -> "EquivariantTransformer":
        e = dict(cfg.extra or {})
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf, cutoff=cfg.cutoff,
                   num_heads=int(e.get("num_heads", 8)), radial_basis=str(e.get("radial_basis", "expnorm")),
                   trainable_rbf=bool(e.get("trainable_rbf", False)), activation=str(e.get("activation", "silu")),
                   attn_activation=str(e.get("attn_activation", "silu")),
                   neighbor_embedding=bool(e.get("neighbor_embedding", True)),
                   distance_influence=str(e.get("distance_influence", "both")),
                   vector_cutoff=bool(e.get("vector_cutoff", True)), n_elements=int(e.get("n_elements", 100)),
                   energy_shift=float(e.get("energy_shift", 0.0)), energy_scale=float(e.get("energy_scale", 1.0)),
                   species=e.get("species"), atomic_energies=e.get("atomic_energies"))
