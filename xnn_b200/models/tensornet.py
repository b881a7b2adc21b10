"""TensorNet (Simeon & De Fabritiis 2023): Cartesian rank-2 tensor message passing.

Per atom the features are ``F`` 3x3 tensors ``X = I 1 + A + S`` (scalar, skew, traceless
symmetric parts). Layout and parameter names follow the reference
(``src/xnn/gnn/models/tensornet.py:79-847``): the embedding builds ``X`` from the neighbour
directions weighted by a pair embedding of both species and three radial projections; each
interaction normalises ``X``, mixes its parts, sums messages ``f_ij (I_j, A_j, S_j)`` (self
pairs included), forms ``C = YM + MY`` (O(3)) or ``2 YM`` (SO(3)), mixes again and updates
``X <- X + dX + dX^2``; the readout takes ``(|I|^2, |A|^2, |S|^2)`` through a LayerNorm and a
linear layer, then an MLP. Edge vectors are ``pos[i] - pos[j]`` (receiver minus sender).

Evaluation plan (same numbers as the part-by-part formulas): the three channel linears of a
tensor's parts commute with the split into parts, so they run as one tensor-core product over
all nine entries, and the split / recombination is one constant per-entry linear map
(:class:`~xnn_b200.ops.tensornet_ops.LinearMap`); messages and the embedding sum onto the atoms
in one kernel each over compact rows, and the per-atom 3x3 products are one kernel
(``csrc/tensornet.cu``). Every piece differentiates to any order (force and stress training).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from ..data import AtomicGraph
from ..nn import CosineCutoff, make_radial_basis
from ..nn.blocks import GatedMLP, make_activation
from ..ops import gemm
from ..ops.scatter import refresh_ghosts
from ..ops.tensornet_ops import (EMBEDDING_FULL, FULL_FROM_COMPACT, RECOMPOSE, Y_AND_COMPACT, TensorPlan,
                                 embedding, geometry_rows, kernels_enabled, matmul3, messages)
from .base import InteratomicPotential
from .fast import AutoPolicy, choose, resolve_use_fast
from .registry import register_model

_READOUTS = ("mlp", "gated")
_GROUPS = ("O(3)", "SO(3)")


def decompose(t: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
    skew = 0.5 * (t - t.transpose(1, 2))
    scalar = t.diagonal(dim1=1, dim2=2).mean(-1)
    eye = torch.eye(3, dtype=t.dtype, device=t.device)
    sym = t - skew - scalar[:, None, None, :] * eye[None, :, :, None]
    return scalar, skew, sym


def frobenius(t: Tensor) -> Tensor:
    return (t * t).sum(dim=(1, 2))


def tensor_matmul(a: Tensor, b: Tensor) -> Tensor:
    """Per atom and channel 3x3 products (one kernel on CUDA, differentiable to any order)."""
    return matmul3(a, b)


class TensorEmbedding(nn.Module):
    def __init__(self, n_features: int, n_rbf: int, n_elements: int, activation: str):
        super().__init__()
        self.n_features = n_features
        self.distance_proj1 = nn.Linear(n_rbf, n_features)
        self.distance_proj2 = nn.Linear(n_rbf, n_features)
        self.distance_proj3 = nn.Linear(n_rbf, n_features)
        self.emb = nn.Embedding(n_elements, n_features)
        self.emb2 = nn.Linear(2 * n_features, n_features)
        self.act = make_activation(activation)
        self.linears_tensor = nn.ModuleList([nn.Linear(n_features, n_features, bias=False) for _ in range(3)])
        self.linears_scalar = nn.ModuleList([nn.Linear(n_features, 2 * n_features),
                                             nn.Linear(2 * n_features, 3 * n_features)])
        self.init_norm = nn.LayerNorm(n_features)

    def forward(self, z: Tensor, src: Tensor, dst: Tensor, cut: Tensor, unit: Tensor, rbf: Tensor,
                plan: Optional[TensorPlan] = None) -> Tensor:
        n, nf = z.shape[0], self.n_features
        if plan is None:
            plan = TensorPlan.build(src, dst, n)
        emb = self.emb(z)
        # emb2 on [emb_i | emb_j] splits into two per-atom products gathered to the pairs
        w_i, w_j = self.emb2.weight[:, :nf], self.emb2.weight[:, nf:]
        pair = (emb @ w_i.t()).index_select(0, dst) + F.linear(emb, w_j, self.emb2.bias).index_select(0, src)
        w = cut.unsqueeze(-1) * pair
        # the three radial projections as one product
        proj = gemm.matmul(rbf, torch.cat([self.distance_proj1.weight, self.distance_proj2.weight,
                                           self.distance_proj3.weight], 0).t()) + torch.cat(
            [self.distance_proj1.bias, self.distance_proj2.bias, self.distance_proj3.bias])
        a = w.unsqueeze(1) * proj.view(-1, 3, nf)
        rows = embedding(a, geometry_rows(unit), plan)
        X = EMBEDDING_FULL(rows).view(n, 3, 3, nf)          # scalar 1 + skew(v) + traceless sym
        norm = self.init_norm(frobenius(X))
        for lin in self.linears_scalar:
            norm = self.act(lin(norm))
        # the part linears commute with the split into parts: one product for all three, the
        # norm factors per part, then the parts recombined
        G = _tensor_products(X, self.linears_tensor[0], self.linears_tensor[1], self.linears_tensor[2])
        G = G.view(n, 9, 3, nf) * norm.view(n, 1, 3, nf)
        return RECOMPOSE(G.reshape(n, 27, nf)).view(n, 3, 3, nf)


def _tensor_products(X: Tensor, l0: nn.Linear, l1: nn.Linear, l2: nn.Linear) -> Tensor:
    """``[X W_0^T | X W_1^T | X W_2^T]`` over every matrix entry of ``X (n, 3, 3, F)``: one product
    on the tensor cores for the three channel linears (bias-free), as ``(n, 27, F)`` rows
    ``entry * 3 + part``."""
    n, nf = X.shape[0], X.shape[-1]
    W = torch.cat([l0.weight, l1.weight, l2.weight], 0).t()
    return gemm.matmul(X.reshape(n * 9, nf), W).view(n, 27, nf)


def _edge_linear(x: Tensor, lin: nn.Linear) -> Tensor:
    """``lin(x)`` for per-pair rows: the tensor-core product (3xTF32, float32 accuracy) when the
    rows are many, differentiable to any order."""
    return gemm.matmul(x, lin.weight.t()) + lin.bias


class Interaction(nn.Module):
    def __init__(self, n_features: int, n_rbf: int, activation: str, o3: bool):
        super().__init__()
        self.n_features = n_features
        self.o3 = o3
        self.act = make_activation(activation)
        self.linears_scalar = nn.ModuleList([nn.Linear(n_rbf, n_features), nn.Linear(n_features, 2 * n_features),
                                             nn.Linear(2 * n_features, 3 * n_features)])
        self.linears_tensor = nn.ModuleList([nn.Linear(n_features, n_features, bias=False) for _ in range(6)])

    def forward(self, X: Tensor, plan: TensorPlan, cut: Tensor, rbf: Tensor, q: Tensor) -> Tensor:
        n, F = X.shape[0], self.n_features
        f = rbf
        for lin in self.linears_scalar:
            f = self.act(_edge_linear(f, lin))
        filters = (f * cut.unsqueeze(-1)).reshape(-1, 3, F)
        X = X / (frobenius(X) + 1.0)[:, None, None, :]
        # channel linears of the parts as one product, then Y and the compact rows of its parts
        Y, rows = Y_AND_COMPACT(_tensor_products(X, *self.linears_tensor[:3]))
        Y = Y.view(n, 3, 3, F)
        msg = FULL_FROM_COMPACT(messages(filters, rows, plan)).view(n, 3, 3, F)
        cs = (1.0 + 0.1 * q)[:, None, None, None]
        C = cs * (tensor_matmul(Y, msg) + tensor_matmul(msg, Y)) if self.o3 else 2.0 * tensor_matmul(Y, msg)
        C = C / (frobenius(C) + 1.0)[:, None, None, :]
        dX = RECOMPOSE(_tensor_products(C, *self.linears_tensor[3:])).view(n, 3, 3, F)
        return X + dX + cs * tensor_matmul(dX, dX)


@register_model("tensornet")
class TensorNet(InteratomicPotential):
    head_modules = ("readout", "atom_ref")
    refreshes_ghosts = True
    readout_extra_inputs = 0

    def __init__(self, n_features: int = 128, n_interactions: int = 2, n_rbf: int = 32, cutoff: float = 4.5,
                 radial_basis: str = "expnorm", trainable_rbf: bool = False, activation: str = "silu",
                 equivariance_group: str = "O(3)", n_elements: int = 128, energy_shift: float = 0.0,
                 energy_scale: float = 1.0, species=None, atomic_energies=None, readout: str = "mlp",
                 readout_hidden=None, self_pairs: bool = True, rbf_max: Optional[float] = None,
                 gamma: Optional[float] = None):
        super().__init__()
        if readout not in _READOUTS:
            raise ValueError(f"readout must be one of {_READOUTS}")
        if equivariance_group not in _GROUPS:
            raise ValueError(f"equivariance_group must be one of {_GROUPS}")
        self.cutoff = float(cutoff)
        if species is not None:
            self.species = [int(z) for z in species]
        self.n_features = n_features
        self.node_feature_dim = n_features
        self.n_interactions = n_interactions
        self.equivariance_group = equivariance_group
        span = float(rbf_max) if rbf_max is not None and radial_basis == "gaussian" else cutoff
        self.rbf = make_radial_basis(radial_basis, n_rbf, span, trainable_rbf, gamma=gamma)
        self.cutoff_fn = CosineCutoff(cutoff)
        self.tensor_embedding = TensorEmbedding(n_features, n_rbf, n_elements, activation)
        self.layers = nn.ModuleList([Interaction(n_features, n_rbf, activation, equivariance_group == "O(3)")
                                     for _ in range(n_interactions)])
        self.out_norm = nn.LayerNorm(3 * n_features)
        self.linear = nn.Linear(3 * n_features, n_features)
        self.act = make_activation(activation)
        self.self_pairs = bool(self_pairs)
        self.use_fast = "auto"
        self.activate_features = readout == "mlp"
        n_in = n_features + self.readout_extra_inputs
        if readout_hidden is None:
            readout_hidden = (n_features // 2,) if readout == "mlp" else (n_in, n_features, n_features)
        sizes = [n_in, *[int(h) for h in readout_hidden], 1]
        if readout == "mlp":
            mods = []
            for a, b in zip(sizes[:-1], sizes[1:]):
                mods += [nn.Linear(a, b), make_activation(activation)]
            self.readout = nn.Sequential(*mods[:-1])
        else:
            self.readout = GatedMLP(sizes, activation)
        for mod in self.readout.modules():
            if isinstance(mod, nn.Linear):
                nn.init.xavier_uniform_(mod.weight)
                nn.init.zeros_(mod.bias)
        self.register_buffer("energy_scale", torch.tensor(float(energy_scale)))
        self.register_buffer("energy_shift", torch.tensor(float(energy_shift)))
        self.atom_ref = nn.Embedding(n_elements, 1)
        nn.init.zeros_(self.atom_ref.weight)
        if atomic_energies is not None:
            if species is None:
                raise ValueError("species is required to map atomic_energies")
            self.set_atomic_energies(species, atomic_energies)

    #: ``"auto"``: the kernels on any CUDA input (faster from the smallest batches measured on)
    AUTO_POLICY = AutoPolicy()

    def set_use_fast(self, use_fast) -> "TensorNet":
        """``False``: the message sums, embeddings and 3 x 3 products run their PyTorch formulas
        also on the GPU; ``True`` / ``"auto"``: the sm_100a kernels on CUDA inputs."""
        self.use_fast = resolve_use_fast(use_fast)
        return self

    def set_atomic_energies(self, species, values) -> None:
        with torch.no_grad():
            self.atom_ref.weight[torch.as_tensor(list(species)), 0] = torch.as_tensor(
                values, dtype=self.atom_ref.weight.dtype)

    def set_energy_scale_shift(self, scale: float, shift: float) -> None:
        self.energy_scale.fill_(float(scale))
        self.energy_shift.fill_(float(shift))

    def receptive_field(self) -> float:
        return max(1, self.n_interactions) * self.cutoff

    def _pairs(self, n_atoms: int, edge_index: Tensor, edge_vec: Tensor):
        """``(src, dst, length, direction)`` of the edges, followed (with ``self_pairs``) by one
        zero-length loop per atom, which carries the atom's own embedding into the messages."""
        length = edge_vec.norm(dim=-1)
        direction = edge_vec / length.clamp(min=1e-12)[:, None]
        src, dst = edge_index.unbind(0)
        if not self.self_pairs:
            return src, dst, length, direction
        ids = torch.arange(n_atoms, dtype=edge_index.dtype, device=edge_index.device)
        return (torch.cat((src, ids)), torch.cat((dst, ids)), F.pad(length, (0, n_atoms)),
                F.pad(direction, (0, 0, 0, n_atoms)))

    def tensors(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor, total_charge: Tensor) -> Tensor:
        """Per-atom 3 x 3 tensor features after the embedding and every interaction."""
        src, dst, length, direction = self._pairs(atomic_numbers.shape[0], edge_index, edge_vec)
        fc, basis = self.cutoff_fn(length), self.rbf(length)
        plan = TensorPlan.build(src, dst, atomic_numbers.shape[0])
        covered = edge_vec.dtype in (torch.float32, torch.float64) and self.n_features <= 128
        fast = choose(getattr(self, "use_fast", "auto"), covered, self.AUTO_POLICY, edge_vec.device,
                      edge_vec.dtype, int(src.shape[0]))
        with kernels_enabled(fast):
            feats = self.tensor_embedding(atomic_numbers, src, dst, fc, direction, basis, plan)
            for layer in self.layers:
                feats = layer(refresh_ghosts(feats), plan, fc, basis, total_charge)
        return feats

    def _features(self, X: Tensor) -> Tensor:
        scalar, skew, sym = decompose(X)
        x = torch.cat([3.0 * scalar * scalar, frobenius(skew), frobenius(sym)], -1)
        x = self.linear(self.out_norm(x))
        return self.act(x) if self.activate_features else x

    def _energy(self, x: Tensor, atomic_numbers: Tensor) -> Tensor:
        return (self.energy_scale * self.readout(x).squeeze(-1) + self.energy_shift
                + self.atom_ref(atomic_numbers).squeeze(-1))

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        q = torch.zeros(atomic_numbers.shape[0], dtype=edge_vec.dtype, device=edge_vec.device)
        x = self._features(self.tensors(atomic_numbers, edge_index, edge_vec, q))
        return x, self._energy(x, atomic_numbers)

    def node_energy(self, atomic_numbers, edge_index, edge_vec):
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> dict:
        vec = data.edge_vectors()
        q = data.total_charge
        qa = (q.index_select(0, data.batch).to(vec.dtype) if q is not None
              else torch.zeros(data.num_nodes, dtype=vec.dtype, device=vec.device))
        x = self._features(self.tensors(data.atomic_numbers, data.edge_index, vec, qa))
        ne = self._energy(x, data.atomic_numbers)
        return {"node_energy": ne, "energy": self.aggregate_energy(ne, data), "node_features": x}

    @classmethod
    def from_config(cls, cfg) -> "TensorNet":
        from ..config.coerce import coerce_per_species, coerce_species
        extra = dict(cfg.extra or {})
        species = coerce_species(extra.get("species")) if extra.get("species") is not None else None
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf,
                   cutoff=cfg.cutoff, radial_basis=str(extra.get("radial_basis", "expnorm")),
                   trainable_rbf=bool(extra.get("trainable_rbf", False)),
                   activation=str(extra.get("activation", "silu")),
                   equivariance_group=str(extra.get("equivariance_group", "O(3)")),
                   n_elements=int(extra.get("n_elements", 128)),
                   energy_shift=float(extra.get("energy_shift", 0.0)),
                   energy_scale=float(extra.get("energy_scale", 1.0)), species=species,
                   atomic_energies=coerce_per_species(extra.get("atomic_energies"), species or [],
                                                      "atomic_energies"),
                   readout=str(extra.get("readout", "mlp")), readout_hidden=extra.get("readout_hidden"),
                   self_pairs=bool(extra.get("self_pairs", True)),
                   rbf_max=None if extra.get("rbf_max") is None else float(extra["rbf_max"]),
                   gamma=None if extra.get("gamma") is None else float(extra["gamma"]))
