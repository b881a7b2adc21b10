"""SchNet (Schuett et al., J. Chem. Phys. 148, 241722 (2018)).

Architecture and parameter names follow the reference's ``src/xnn/gnn/models/schnet.py:84-560``
(``embedding``, ``rbf``, ``interactions[k].{lin_in, cfconv.filter_net, lin_mid, lin_out}``,
``readout``, ``energy_scale`` / ``energy_shift`` buffers, ``atom_ref``), so checkpoints load in
either framework. On CUDA the continuous-filter convolution ``sum_j x_j * W(r_ij)`` runs on the
block-per-atom message-pass kernels of ``csrc/conv.cu`` (one degree, unit angular factor) when
the edges are grouped by receiver; otherwise on PyTorch index operations.
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from ..data.atomic_graph import AtomicGraph
from ..nn.cutoff import CosineCutoff
from ..nn.radial import make_radial_basis
from ..ops.scatter import scatter_sum
from .base import InteratomicPotential
from .fast import AutoPolicy, choose, resolve_use_fast
from .registry import register_model

MAX_Z = 100


class ShiftedSoftplus(nn.Module):
    def forward(self, x: Tensor) -> Tensor:
        return F.softplus(x) - math.log(2.0)


def make_activation(name: str) -> nn.Module:
    return {"silu": nn.SiLU(), "ssp": ShiftedSoftplus(), "tanh": nn.Tanh(), "relu": nn.ReLU(),
            "linear": nn.Identity()}[name]


class _CFConv(nn.Module):
    def __init__(self, n_filters: int, n_rbf: int, output_activation: bool = False):
        super().__init__()
        layers = [nn.Linear(n_rbf, n_filters), ShiftedSoftplus(), nn.Linear(n_filters, n_filters)]
        if output_activation:
            layers.append(ShiftedSoftplus())
        self.filter_net = nn.Sequential(*layers)
        self.n_filters = n_filters

    def forward(self, x: Tensor, edge_index: Tensor, rbf: Tensor, envelope: Optional[Tensor], plan=None) -> Tensor:
        W = self.filter_net(rbf)
        if envelope is not None:
            W = W * envelope[:, None]
        if plan is not None:
            from ..ops import mace_ops as K
            ones = torch.ones(W.shape[0], 1, dtype=W.dtype, device=W.device)
            return K.conv(x, W[:, None, :].contiguous(), ones, plan)[0]
        src, dst = edge_index[0], edge_index[1]
        return scatter_sum(x[src] * W, dst, x.shape[0])


class _Interaction(nn.Module):
    def __init__(self, n_features: int, n_rbf: int, n_filters: int, filter_output_activation: bool = False,
                 input_bias: bool = False):
        super().__init__()
        self.lin_in = nn.Linear(n_features, n_filters, bias=input_bias)
        self.cfconv = _CFConv(n_filters, n_rbf, filter_output_activation)
        self.lin_mid = nn.Linear(n_filters, n_features)
        self.lin_out = nn.Linear(n_features, n_features)

    def forward(self, x, edge_index, rbf, envelope, plan=None) -> Tensor:
        h = self.cfconv(self.lin_in(x), edge_index, rbf, envelope, plan)
        return self.lin_out(F.softplus(self.lin_mid(h)) - math.log(2.0))


@register_model("schnet")
class SchNet(InteratomicPotential):
    head_modules = ("readout", "atom_ref")

    def __init__(self, n_features: int = 128, n_interactions: int = 6, n_rbf: int = 20, cutoff: float = 5.0,
                 radial_basis: str = "gaussian", gamma: Optional[float] = None, cutoff_fn: Optional[str] = "cosine",
                 n_filters: Optional[int] = None, filter_output_activation: bool = False,
                 interaction_input_bias: bool = False, readout_activation: str = "silu",
                 shared_interactions: bool = False, zero_init_readout: bool = False, energy_shift: float = 0.0,
                 energy_scale: float = 1.0, species=None, atomic_energies=None):
        super().__init__()
        if cutoff_fn not in (None, "cosine"):
            raise ValueError(f"cutoff_fn must be None or 'cosine', got {cutoff_fn!r}")
        self.cutoff = float(cutoff)
        if species is not None:
            self.species = [int(z) for z in species]
        self.node_feature_dim = n_features
        self.embedding = nn.Embedding(MAX_Z, n_features)
        self.rbf = make_radial_basis(radial_basis, n_rbf, cutoff, gamma=gamma)
        n_filters = n_features if n_filters is None else n_filters
        shared = _Interaction(n_features, n_rbf, n_filters, filter_output_activation,
                              interaction_input_bias) if shared_interactions else None
        self.interactions = nn.ModuleList([
            shared if shared is not None else _Interaction(n_features, n_rbf, n_filters, filter_output_activation,
                                                           interaction_input_bias)
            for _ in range(n_interactions)])
        self.cutoff_fn = CosineCutoff(cutoff) if cutoff_fn == "cosine" else None
        self.readout = nn.Sequential(nn.Linear(n_features, n_features // 2), make_activation(readout_activation),
                                     nn.Linear(n_features // 2, 1))
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        if zero_init_readout:
            nn.init.zeros_(self.readout[-1].weight)
            nn.init.zeros_(self.readout[-1].bias)
        self.register_buffer("energy_scale", torch.tensor(float(energy_scale)))
        self.register_buffer("energy_shift", torch.tensor(float(energy_shift)))
        self.atom_ref = nn.Embedding(MAX_Z, 1)
        nn.init.zeros_(self.atom_ref.weight)
        if atomic_energies is not None:
            self.set_atomic_energies(species, atomic_energies)
        self.use_fast = "auto"

    #: ``"auto"``: the CSR segment sums on any CUDA input with receiver-sorted edges
    AUTO_POLICY = AutoPolicy()

    def set_use_fast(self, use_fast) -> "SchNet":
        self.use_fast = resolve_use_fast(use_fast)
        return self

    def set_atomic_energies(self, species, values) -> None:
        ae = torch.as_tensor(values, dtype=self.atom_ref.weight.dtype)
        with torch.no_grad():
            self.atom_ref.weight[torch.tensor(list(species)), 0] = ae

    def receptive_field(self) -> float:
        return len(self.interactions) * self.cutoff

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor,
                             plan=None) -> Tuple[Tensor, Tensor]:
        x = self.embedding(atomic_numbers)
        r = torch.linalg.norm(edge_vec, dim=-1)
        rbf = self.rbf(r)
        env = self.cutoff_fn(r) if self.cutoff_fn is not None else None
        for block in self.interactions:
            x = x + block(x, edge_index, rbf, env, plan)
        node_energy = (self.energy_scale * self.readout(x).squeeze(-1) + self.energy_shift
                       + self.atom_ref(atomic_numbers).squeeze(-1))
        return x, node_energy

    def node_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor) -> Tensor:
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        edge_vec = data.edge_vectors()
        plan = None
        if choose(self.use_fast, edge_vec.is_cuda and data.edge_order == "dst", self.AUTO_POLICY, edge_vec.device,
                  edge_vec.dtype, data.num_edges):
            from ..ops.mace_ops import EdgePlan
            plan = EdgePlan.build(data.edge_index, data.num_nodes, assume_dst_sorted=True)
        x, node_energy = self.node_features_energy(data.atomic_numbers, data.edge_index, edge_vec, plan)
        return {"node_energy": node_energy, "energy": self.aggregate_energy(node_energy, data), "node_features": x}

    @classmethod
    def from_config(cls, cfg) -> "SchNet":
        e = dict(cfg.extra or {})
        keys = ("radial_basis", "gamma", "cutoff_fn", "n_filters", "filter_output_activation",
                "interaction_input_bias", "readout_activation", "shared_interactions", "zero_init_readout",
                "energy_shift", "energy_scale", "species", "atomic_energies")
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf,
                   cutoff=cfg.cutoff, **{k: e[k] for k in keys if k in e})
