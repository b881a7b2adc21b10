"""CACE (Cheng, npj Comput. Mater. 2024): the Cartesian atomic cluster expansion.

Edges carry Bessel radials (polynomial envelope) times Cartesian monomials ``x^a y^b z^c`` of the
unit vector times a sender x receiver species embedding; their per-atom sums are mixed by a radial
transform shared per ``l``; the symmetrizer contracts the monomial index into rotational
invariants of body order ``nu <= 4`` (multinomial-weighted products, grouped by ``l`` tuples);
message passes add memory (``M``), radially decaying neighbour features (``Ar``) and the
re-weighted edge basis (``Bchi``); the readout is an MLP plus a linear term on all passes'
invariants. The invariant grouping and its order, options and parameter names follow the
reference (``src/xnn/gnn/models/cace.py``, ``featurizers/cartesian.py``) so that weights
transplant.
"""
from __future__ import annotations

from math import factorial
from typing import List, Optional

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.cutoff import PolynomialCutoff
from ..nn.radial import BesselRBF
from ..ops.scatter import scatter_sum
from .base import GNNPotential
from .registry import register_model

MESSAGE_TYPES = ("M", "Ar", "Bchi")


def lxlylz_list(l_max: int) -> list:
    return [(lx, ly, l - lx - ly) for l in range(l_max + 1) for lx in range(l + 1) for ly in range(l + 1 - lx)]


def multinomial(c) -> int:
    lx, ly, lz = (int(v) for v in c)
    return factorial(lx + ly + lz) // (factorial(lx) * factorial(ly) * factorial(lz))


class CartesianAngularBasis(nn.Module):
    """Monomials ``u_x^a u_y^b u_z^c`` with ``a + b + c <= l_max``, each from a parent monomial."""

    def __init__(self, l_max: int):
        super().__init__()
        self.l_max = l_max
        self.lxlylz = lxlylz_list(l_max)
        self.n_angular = len(self.lxlylz)
        index = {c: i for i, c in enumerate(self.lxlylz)}
        self._steps = []
        for c in self.lxlylz[1:]:
            k = max(range(3), key=lambda i: c[i])
            parent = list(c)
            parent[k] -= 1
            self._steps.append((index[tuple(parent)], k))
        self.register_buffer("l_of_entry", torch.tensor([sum(c) for c in self.lxlylz]), persistent=False)

    def forward(self, unit: Tensor) -> Tensor:
        feats = [torch.ones_like(unit[:, 0])]
        for p, k in self._steps:
            feats.append(feats[p] * unit[:, k])
        return torch.stack(feats, 1)


def _groups(nu: int, l_max: int) -> dict:
    """Contraction terms per invariant (``l``-tuple key, insertion-ordered), each ``(monomials, weight)``."""
    out: dict = {}
    rng = range(l_max + 1)
    trip = [(x, y, z) for x in rng for y in rng for z in rng]
    if nu == 2:
        for c in lxlylz_list(l_max):
            if sum(c) >= 1:
                out.setdefault(sum(c), []).append(((c, c), multinomial(c)))
    elif nu == 3:
        for c1 in trip:
            l1 = sum(c1)
            if not 0 < l1 <= l_max:
                continue
            for c2 in trip:
                l2 = sum(c2)
                if not l1 <= l2 <= l_max:
                    continue
                c3 = tuple(a + b for a, b in zip(c1, c2))
                if sum(c3) <= l_max:
                    out.setdefault((l1, l2), []).append(((c1, c2, c3), multinomial(c1) * multinomial(c2)))
    elif nu == 4:
        for c1 in trip:
            l1 = sum(c1)
            if not 0 < l1 <= l_max:
                continue
            for c2 in trip:
                l2 = sum(c2)
                if not l1 < l2 <= l_max:
                    continue
                for dd in trip:
                    if sum(dd) < 1:
                        continue
                    c3 = tuple(a + b for a, b in zip(c1, dd))
                    c4 = tuple(a + b for a, b in zip(c2, dd))
                    if sum(c3) <= l_max and sum(c4) <= l_max:
                        out.setdefault((l1, l2, sum(dd)), []).append(
                            ((c1, c2, c3, c4), multinomial(c1) * multinomial(c2) * multinomial(dd)))
    return out


class _Symmetrizer(nn.Module):
    def __init__(self, max_nu: int, l_max: int):
        super().__init__()
        if not 1 <= max_nu <= 4:
            raise ValueError(f"max_nu must be in 1..4, got {max_nu}")
        self.max_nu, self.l_max = max_nu, l_max
        index = {c: i for i, c in enumerate(lxlylz_list(l_max))}
        self.n_features = 1
        self._orders = []
        for nu in (2, 3, 4):
            idx, pref, out = [], [], []
            if nu <= max_nu:
                groups = _groups(nu, l_max)
                for g, terms in enumerate(groups.values()):
                    for combo, w in terms:
                        idx.append([index[c] for c in combo])
                        pref.append(float(w))
                        out.append(self.n_features + g)
                self.n_features += len(groups)
            self.register_buffer(f"_idx{nu}", torch.tensor(idx, dtype=torch.long).reshape(-1, nu), persistent=False)
            self.register_buffer(f"_pref{nu}", torch.tensor(pref), persistent=False)
            self.register_buffer(f"_out{nu}", torch.tensor(out, dtype=torch.long), persistent=False)

    def forward(self, a: Tensor) -> Tensor:
        n, r, _, c = a.shape
        out = a.new_zeros(n, r, self.n_features, c)
        out[:, :, 0, :] = a[:, :, 0, :]
        for nu in (2, 3, 4):
            idx = getattr(self, f"_idx{nu}")
            if idx.numel():
                prods = a[:, :, idx, :].prod(3) * getattr(self, f"_pref{nu}").to(a.dtype)[None, None, :, None]
                out = out.index_add(2, getattr(self, f"_out{nu}"), prods)
        return out


class _SharedRadialTransform(nn.Module):
    def __init__(self, l_of_entry: Tensor, n_rbf: int, n_radial: int, channels: int):
        super().__init__()
        self.weight = nn.Parameter(torch.rand(int(l_of_entry.max()) + 1, n_rbf, n_radial, channels))
        self.register_buffer("l_of_entry", l_of_entry.clone(), persistent=False)

    def forward(self, a: Tensor) -> Tensor:
        return torch.einsum("nrac,armc->nmac", a, self.weight[self.l_of_entry])


class _NodeMemory(nn.Module):
    def __init__(self, l_of_entry: Tensor, n_radial: int, channels: int):
        super().__init__()
        self.memory_coef = nn.Parameter(torch.full((int(l_of_entry.max()) + 1, n_radial, channels), 0.25))
        self.register_buffer("l_of_entry", l_of_entry.clone(), persistent=False)

    def forward(self, a: Tensor) -> Tensor:
        return a * self.memory_coef[self.l_of_entry].permute(1, 0, 2)


class _MessageAr(nn.Module):
    def __init__(self, l_of_entry: Tensor, cutoff: float, n_radial: int, channels: int):
        super().__init__()
        lm = int(l_of_entry.max())
        self.prefactor = nn.Parameter(torch.rand(lm + 1, n_radial, channels))
        self.inv_r0 = nn.Parameter((torch.rand(lm + 1, n_radial, channels) + 0.5) / cutoff)
        self.register_buffer("l_of_entry", l_of_entry.clone(), persistent=False)

    def forward(self, a: Tensor, lengths: Tensor, envelope: Tensor, sender: Tensor) -> Tensor:
        decay = torch.exp(-lengths[:, None, None, None] * self.inv_r0) * self.prefactor * envelope[:, None, None, None]
        # (E, l, r, c) -> per monomial entry through its l
        return a.index_select(0, sender) * decay[:, self.l_of_entry].transpose(1, 2)


class _MessageBchi(nn.Module):
    def __init__(self, n_b_flat: int):
        super().__init__()
        self.h = nn.Linear(n_b_flat, 1)

    def forward(self, b: Tensor, edge_attr: Tensor, sender: Tensor) -> Tensor:
        return edge_attr * self.h(b.flatten(1))[sender][:, :, None, None]


class _CaceInteraction(nn.Module):
    def __init__(self, l_of_entry, cutoff, n_radial, channels, n_b_flat, message_types, mp_norm):
        super().__init__()
        self.mp_norm = mp_norm
        self.memory = _NodeMemory(l_of_entry, n_radial, channels) if "M" in message_types else None
        self.message_ar = _MessageAr(l_of_entry, cutoff, n_radial, channels) if "Ar" in message_types else None
        self.message_bchi = _MessageBchi(n_b_flat) if "Bchi" in message_types else None

    def forward(self, a: Tensor, bchi: Optional[Tensor], lengths: Tensor, envelope: Tensor, edge_index: Tensor):
        new = torch.zeros_like(a)
        if self.message_ar is not None:
            new = new + scatter_sum(self.message_ar(a, lengths, envelope, edge_index[0]), edge_index[1], a.shape[0])
        if bchi is not None:
            new = new + bchi
        new = new * self.mp_norm
        if self.memory is not None:
            new = new + self.memory(a)
        return new


@register_model("cace")
class CACE(GNNPotential):
    head_modules = ("readout_mlp", "readout_linear", "atom_ref")

    def __init__(self, species, cutoff: float = 5.5, n_atom_basis: int = 3, n_rbf: int = 8,
                 n_radial_basis: Optional[int] = None, max_l: int = 3, max_nu: int = 3, num_message_passing: int = 1,
                 message_types=("M", "Ar", "Bchi"), embed_receiver_nodes: bool = False, avg_num_neighbors: float = 10.0,
                 num_polynomial_cutoff: int = 6, trainable_rbf: bool = True, readout_hidden=None,
                 atomic_energies=None):
        super().__init__(species, cutoff)
        message_types = tuple(message_types)
        unknown = set(message_types) - set(MESSAGE_TYPES)
        if unknown:
            raise ValueError(f"unknown message types {sorted(unknown)}; choose from {MESSAGE_TYPES}")
        if num_message_passing > 0 and not message_types:
            raise ValueError("message_types must not be empty when num_message_passing > 0")
        self.n_atom_basis, self.channels = n_atom_basis, n_atom_basis ** 2
        self.n_rbf, self.n_radial_basis = n_rbf, n_radial_basis or n_rbf
        self.max_l, self.max_nu, self.message_types = max_l, max_nu, message_types
        self.mp_norm = avg_num_neighbors ** -0.5
        self.embed_sender = nn.Parameter(nn.init.xavier_uniform_(torch.empty(len(self.species), n_atom_basis)))
        self.embed_receiver = (nn.Parameter(nn.init.xavier_uniform_(torch.empty(len(self.species), n_atom_basis)))
                               if embed_receiver_nodes else self.embed_sender)
        self.rbf = BesselRBF(n_rbf, cutoff, trainable=trainable_rbf)
        self.envelope = PolynomialCutoff(cutoff, p=num_polynomial_cutoff)
        self.angular = CartesianAngularBasis(max_l)
        le = self.angular.l_of_entry
        self.radial_transform = _SharedRadialTransform(le, n_rbf, self.n_radial_basis, self.channels)
        self.symmetrizer = _Symmetrizer(max_nu, max_l)
        self.n_b_features = self.symmetrizer.n_features
        n_b_flat = self.n_radial_basis * self.n_b_features * self.channels
        self.interactions = nn.ModuleList([_CaceInteraction(le, cutoff, self.n_radial_basis, self.channels, n_b_flat,
                                                            message_types, self.mp_norm)
                                           for _ in range(num_message_passing)])
        feat = n_b_flat * (num_message_passing + 1)
        self.node_feature_dim = feat
        widths = [feat] + list(readout_hidden or [32, 16])
        layers: List[nn.Module] = []
        for a, b in zip(widths[:-1], widths[1:]):
            layers += [nn.Linear(a, b), nn.SiLU()]
        layers.append(nn.Linear(widths[-1], 1))
        self.readout_mlp = nn.Sequential(*layers)
        self.readout_linear = nn.Linear(feat, 1)
        if atomic_energies is not None:
            self.set_atomic_energies(atomic_energies)

    def receptive_field(self) -> float:
        return (len(self.interactions) + 1) * self.cutoff

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        n = atomic_numbers.shape[0]
        sender, receiver = edge_index[0], edge_index[1]
        lengths = torch.linalg.norm(edge_vec, dim=-1)
        unit = edge_vec / (lengths + 1e-9).unsqueeze(-1)
        one_hot = self.node_attr(atomic_numbers)
        envelope = self.envelope(lengths)
        radial = self.rbf(lengths) * envelope.unsqueeze(-1)
        angular = self.angular(unit)
        ts = (one_hot @ self.embed_sender).index_select(0, sender)
        tr = (one_hot @ self.embed_receiver).index_select(0, receiver)
        edge_type = (ts.unsqueeze(2) * tr.unsqueeze(1)).flatten(1)
        edge_attr = radial[:, :, None, None] * angular[:, None, :, None] * edge_type[:, None, None, :]
        a = self.radial_transform(scatter_sum(edge_attr, receiver, n))
        feats = [self.symmetrizer(a)]
        for inter in self.interactions:
            bchi = None
            if inter.message_bchi is not None:
                bchi = self.radial_transform(scatter_sum(inter.message_bchi(feats[-1], edge_attr, sender), receiver, n))
            a = inter(a, bchi, lengths, envelope, edge_index)
            feats.append(self.symmetrizer(a))
        x = torch.stack(feats, -1).flatten(1)
        e = self.readout_mlp(x) + self.readout_linear(x)
        return x, e.squeeze(-1) + self.atom_ref(atomic_numbers).squeeze(-1)

    def node_energy(self, atomic_numbers, edge_index, edge_vec):
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> dict:
        x, e = self.node_features_energy(data.atomic_numbers, data.edge_index, data.edge_vectors())
        return {"node_energy": e, "energy": self.aggregate_energy(e, data), "node_features": x}

    @classmethod
    def from_config(cls, cfg) -> "CACE":
        e = dict(cfg.extra or {})
        keys = ("n_radial_basis", "max_l", "max_nu", "message_types", "embed_receiver_nodes", "avg_num_neighbors",
                "num_polynomial_cutoff", "trainable_rbf", "readout_hidden", "atomic_energies")
        species = [int(z) for z in e.get("species") or [1, 6, 7, 8]]
        return cls(species=species, cutoff=cfg.cutoff, n_atom_basis=cfg.n_features, n_rbf=cfg.n_rbf,
                   num_message_passing=cfg.n_interactions, **{k: e[k] for k in keys if k in e})
