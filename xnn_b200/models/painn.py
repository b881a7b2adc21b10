"""PaiNN (Schuett, Unke & Gastegger, ICML 2021): equivariant message passing with scalar and
vector features.

Architecture and parameter names follow the reference's ``src/xnn/gnn/models/painn.py:117-760``
(``embedding``, ``rbf``, one stacked ``filters`` layer for every block, ``interactions[k].message.phi``,
``interactions[k].update.{lin_v, net}``, ``readout``, ``energy_scale`` / ``energy_shift``,
``atom_ref``), including its edge-direction convention (the paper's ``r_ij = r_j - r_i`` is the
negative of the edge vector).
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
from torch import Tensor, nn

from ..data.atomic_graph import AtomicGraph
from ..nn.cutoff import CosineCutoff
from ..nn.radial import make_radial_basis
from ..ops.scatter import scatter_sum
from .base import InteratomicPotential
from .registry import register_model

MAX_Z = 100


class _Message(nn.Module):
    def __init__(self, n_features: int, vector_propagation: bool = True, vectors: bool = True, phi=None):
        super().__init__()
        self.n_features = n_features
        self.vectors = vectors
        self.vector_propagation = vectors and vector_propagation
        self.n_parts = 1 + int(vectors) + int(self.vector_propagation)
        self.phi = phi if phi is not None else nn.Sequential(
            nn.Linear(n_features, n_features), nn.SiLU(), nn.Linear(n_features, self.n_parts * n_features))

    def forward(self, s: Tensor, v: Tensor, W: Tensor, direction: Tensor, edge_index: Tensor):
        src, dst = edge_index[0], edge_index[1]
        n = s.shape[0]
        parts = torch.split(self.phi(s)[src] * W, self.n_features, dim=-1)
        ds = scatter_sum(parts[0], dst, n)
        if not self.vectors:
            return ds, torch.zeros_like(v)
        dv = parts[self.n_parts - 1][:, None, :] * direction[:, :, None]
        if self.vector_propagation:
            dv = dv + parts[1][:, None, :] * v[src]
        return ds, scatter_sum(dv, dst, n)


class _Update(nn.Module):
    def __init__(self, n_features: int, epsilon: float = 1e-8, scalar_product: bool = True, vectors: bool = True):
        super().__init__()
        self.n_features = n_features
        self.vectors = vectors
        self.scalar_product = vectors and scalar_product
        self.n_parts = 1 + int(vectors) + int(self.scalar_product)
        self.lin_v = nn.Linear(n_features, 2 * n_features, bias=False) if vectors else None
        self.net = nn.Sequential(nn.Linear((1 + int(vectors)) * n_features, n_features), nn.SiLU(),
                                 nn.Linear(n_features, self.n_parts * n_features))
        self.epsilon = epsilon

    def forward(self, s: Tensor, v: Tensor):
        if not self.vectors:
            return self.net(s), torch.zeros_like(v)
        uv, vv = torch.split(self.lin_v(v), self.n_features, dim=-1)
        norm = torch.sqrt((vv * vv).sum(dim=1) + self.epsilon)
        parts = torch.split(self.net(torch.cat([s, norm], dim=-1)), self.n_features, dim=-1)
        dv = parts[0][:, None, :] * uv
        ds = parts[self.n_parts - 1]
        if self.scalar_product:
            ds = ds + parts[1] * (uv * vv).sum(dim=1)
        return ds, dv


class _Interaction(nn.Module):
    def __init__(self, message: _Message, update: _Update):
        super().__init__()
        self.message = message
        self.update = update

    def forward(self, s, v, W, direction, edge_index):
        ds, dv = self.message(s, v, W, direction, edge_index)
        s, v = s + ds, v + dv
        ds, dv = self.update(s, v)
        return s + ds, v + dv


def _mlp(n_features: int, n_layers: int) -> nn.Sequential:
    widths = [n_features]
    for _ in range(n_layers - 1):
        widths.append(max(1, widths[-1] // 2))
    widths.append(1)
    layers = []
    for i in range(n_layers):
        layers.append(nn.Linear(widths[i], widths[i + 1]))
        if i < n_layers - 1:
            layers.append(nn.SiLU())
    return nn.Sequential(*layers)


@register_model("painn")
class PaiNN(InteratomicPotential):
    head_modules = ("readout", "atom_ref")

    def __init__(self, n_features: int = 128, n_interactions: int = 3, n_rbf: int = 20, cutoff: float = 5.0,
                 radial_basis: str = "gaussian", trainable_rbf: bool = False, shared_filters: bool = False,
                 shared_interactions: bool = False, epsilon: float = 1e-8, scalar_product: bool = True,
                 vector_propagation: bool = True, vector_features: bool = True, energy_shift: float = 0.0,
                 energy_scale: float = 1.0, species=None, atomic_energies=None):
        super().__init__()
        self.cutoff = float(cutoff)
        if species is not None:
            self.species = [int(z) for z in species]
        self.n_features = n_features
        self.node_feature_dim = n_features
        self.shared_filters = shared_filters
        self.embedding = nn.Embedding(MAX_Z, n_features)
        self.rbf = make_radial_basis(radial_basis, n_rbf, cutoff, trainable_rbf,
                                     prefactor=1.0 if radial_basis == "bessel" else None)
        self.cutoff_fn = CosineCutoff(cutoff)
        self.filter_width = (1 + int(vector_features) + int(vector_features and vector_propagation)) * n_features
        self.filters = nn.Linear(n_rbf, (1 if shared_filters else n_interactions) * self.filter_width)
        blocks = []
        for _ in range(n_interactions):
            if shared_interactions and blocks:
                first = blocks[0]
                blocks.append(_Interaction(_Message(n_features, vector_propagation, vector_features,
                                                    phi=first.message.phi), first.update))
            else:
                blocks.append(_Interaction(_Message(n_features, vector_propagation, vector_features),
                                           _Update(n_features, epsilon, scalar_product, vector_features)))
        self.interactions = nn.ModuleList(blocks)
        self.readout = _mlp(n_features, 2)
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        self.register_buffer("energy_scale", torch.tensor(float(energy_scale)))
        self.register_buffer("energy_shift", torch.tensor(float(energy_shift)))
        self.atom_ref = nn.Embedding(MAX_Z, 1)
        nn.init.zeros_(self.atom_ref.weight)
        from ..data.elements import _WEIGHTS
        # standard atomic weights (centre of mass of dipole outputs), kept in the state dict
        self.register_buffer("masses", torch.tensor(_WEIGHTS[:MAX_Z], dtype=torch.float64))
        if atomic_energies is not None:
            with torch.no_grad():
                self.atom_ref.weight[torch.tensor(list(species)), 0] = torch.as_tensor(atomic_energies).to(
                    self.atom_ref.weight)

    def receptive_field(self) -> float:
        return len(self.interactions) * self.cutoff

    def representation(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        r = torch.linalg.norm(edge_vec, dim=-1)
        direction = -edge_vec / r.clamp(min=1e-12)[:, None]
        W = self.filters(self.rbf(r)) * self.cutoff_fn(r)[:, None]
        filters = torch.split(W, self.filter_width, dim=-1)
        s = self.embedding(atomic_numbers)
        v = torch.zeros((s.shape[0], 3, s.shape[1]), dtype=s.dtype, device=s.device)
        for k, block in enumerate(self.interactions):
            s, v = block(s, v, filters[k % len(filters)], direction, edge_index)
        return s, v

    def node_features_energy(self, atomic_numbers, edge_index, edge_vec) -> Tuple[Tensor, Tensor]:
        s, _ = self.representation(atomic_numbers, edge_index, edge_vec)
        return s, (self.energy_scale * self.readout(s).squeeze(-1) + self.energy_shift
                   + self.atom_ref(atomic_numbers).squeeze(-1))

    def node_energy(self, atomic_numbers, edge_index, edge_vec) -> Tensor:
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        s, e = self.node_features_energy(data.atomic_numbers, data.edge_index, data.edge_vectors())
        return {"node_energy": e, "energy": self.aggregate_energy(e, data), "node_features": s}

    @classmethod
    def from_config(cls, cfg) -> "PaiNN":
        e = dict(cfg.extra or {})
        keys = ("radial_basis", "trainable_rbf", "shared_filters", "shared_interactions", "epsilon",
                "scalar_product", "vector_propagation", "vector_features", "energy_shift", "energy_scale",
                "species", "atomic_energies")
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf,
                   cutoff=cfg.cutoff, **{k: e[k] for k in keys if k in e})
