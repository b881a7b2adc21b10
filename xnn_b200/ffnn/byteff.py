"""ByteFF: a classical force field whose parameters are predicted from the molecular graph.

An edge-augmented graph transformer (EGT) embeds each distinct molecule once; a bonded head pools
the atom and bond channels along every bond, angle, proper torsion and improper (both directions,
or the three arms of an improper) and predicts harmonic bond / angle constants and the four-term
Fourier series of each torsion (standardised outputs, a tanh bound, clamped with a straight-
through gradient); a non-bonded head predicts Lennard-Jones ``sigma`` / ``epsilon`` per atom and
charges as bond-charge increments on the class-averaged formal charges (so each molecule keeps its
total charge). An ensemble of ``members`` averages the predictions. The energy is then the
classical one over the bound system: harmonic bonds and angles, torsions ``sum_n k_n [1 + s_n
cos(n phi)]`` (``s = +1`` odd ``n``, ``-1`` even), impropers ``k (1 - cos 2 phi)``, Lennard-Jones
with the arithmetic sigma and geometric epsilon, Coulomb, 1-2 / 1-3 pairs excluded and 1-4 pairs
scaled by ``fudge_lj`` / ``fudge_qq``; every pair of the structure (``cutoff=None``, molecules) or
the neighbour list within a cutoff with a quintic switch (liquids, periodic cells). Hypervalent
P / S centres get fixed stiff bonds and angles at the geometry given as ``reference_positions``
and no torsions. Energies in kcal/mol internally, eV out.

Here the system is bound from explicit molecular graphs (bonds, bond orders and formal charges;
:func:`xnn_b200.featurizers.molgraph.molecular_graph_from_bonds`) rather than perceived by RDKit.
Architecture, output statistics and bounds, parameter names and the energy conventions follow the
reference (``src/xnn/hybnn/models/byteff.py``) so trained weights transplant.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..featurizers.molgraph import MolecularGraph, molecular_graph_from_bonds
from ..models.base import InteratomicPotential
from ..models.egt import MolecularGraphTransformer, class_mean
from ..models.registry import register_model
from ..nn.blocks import MLP
from ..ops.scatter import scatter_sum
from .geometry import geometric_mean, half_edges, pair_vectors, quintic_switch
from .opls import KCAL_TO_EV

COULOMB = 332.0637141491396
TERM_ATOMS = {"bond": 2, "angle": 3, "proper": 4, "improper": 2}
# name: (width, std, mean, lower, upper) of each predicted parameter
HARMONIC = {
    "bond": {"bond_k": (1, 200.0, 700.0, 80.0, 4000.0), "bond_r0": (1, 0.19, 1.3, 0.5, 5.0)},
    "angle": {"angle_k": (1, 60.0, 130.0, 40.0, 1000.0), "angle_d0": (1, 10.0, 120.0, 20.0, 180.0)},
    "proper": {"proper_k": (4, 1.2, 0.4, -20.0, 20.0)},
    "improper": {"improper_k": (1, 3.7, 4.3, 0.0, 20.0)},
}
TWO_WELL = {
    "bond": {"bond_k1": (1, 50.0, 1000.0, 0.0, 4000.0), "bond_k2": (1, 25.0, 500.0, 0.0, 4000.0)},
    "angle": {"angle_k1": (1, 5.0, 100.0, 0.0, 400.0), "angle_k2": (1, 5.0, 100.0, 0.0, 400.0)},
    "proper": {"proper_k": (4, 1.2, 0.4, -20.0, 20.0)},
    "improper": {"improper_k": (1, 3.7, 4.3, 0.0, 40.0)},
}
TWO_WELL_BONDS = (0.5, 4.0)
TWO_WELL_ANGLES = (0.25 * math.pi, 1.05 * math.pi)
HYPERVALENT_K = {"bond": 1000.0, "angle": 278.44}
GRAPH_DEFAULTS = dict(atom_dim=32, feature_dim=8, node_mlp=(64, 256, 2), edge_mlp=(64, 256, 2), hidden=256, layers=4,
                      heads=16, head_dim=16, ffn=(256, 2), out_dim=256, jumping_knowledge="cat", activation="gelu")
TERMS = ("e_bond", "e_angle", "e_torsion", "e_improper", "e_vdw", "e_coulomb", "e_vdw14", "e_coulomb14")


def _mlp(n_in: int, hidden: int, n_out: int, layers: int, activation: str = "gelu", bias: bool = True) -> MLP:
    return MLP([n_in] + [hidden] * (layers - 1) + [n_out], activation, bias=bias)


def _clamp_st(x: Tensor, lo: float, hi: float) -> Tensor:
    """Clamped value, identity gradient (the bound does not stop training)."""
    return x + (torch.clamp(x, lo, hi) - x).detach()


class BondedHead(nn.Module):
    """Per-term parameters from the atom / bond channels pooled along each term."""

    def __init__(self, node_dim: int, edge_dim: int, pre=(256, 256, 3), out=(256, 4), tanh_output: float = 20.0,
                 form: str = "harmonic", activation: str = "gelu"):
        super().__init__()
        if form not in ("harmonic", "two_well"):
            raise ValueError(f"form must be 'harmonic' or 'two_well', got {form!r}")
        self.form, self.tanh_output = form, float(tanh_output)
        self.table = HARMONIC if form == "harmonic" else TWO_WELL
        self.pool = nn.ModuleDict({t: _mlp(a * node_dim + (a - 1) * edge_dim, pre[0], pre[1], pre[2], activation)
                                   for t, a in TERM_ATOMS.items()})
        self.post = nn.ModuleDict({t: _mlp(pre[1], pre[0], pre[1], pre[2], activation) for t in TERM_ATOMS})
        self.out = nn.ModuleDict({p: _mlp(pre[1], out[0], spec[0], out[1], activation)
                                  for t in TERM_ATOMS for p, spec in self.table[t].items()})

    @staticmethod
    def _views(kind: str, x: Tensor, e: Tensor, atoms: Tensor, edges: Tensor) -> List[Tensor]:
        if kind == "improper":
            # the three arms centre -> neighbour
            return [torch.cat([x[atoms[:, 0]], e[edges[:, k]], x[atoms[:, k + 1]]], -1) for k in range(3)]
        seq = []
        for k in range(atoms.shape[1]):
            seq.append(x[atoms[:, k]])
            if k < edges.shape[1]:
                seq.append(e[edges[:, k]])
        return [torch.cat(seq, -1), torch.cat(seq[::-1], -1)]

    def forward(self, x: Tensor, e: Tensor, terms: dict) -> Dict[str, Tensor]:
        params = {}
        for kind in TERM_ATOMS:
            atoms, edges = terms[kind]
            views = self._views(kind, x, e, atoms, edges)
            m = atoms.shape[0]
            pooled = self.pool[kind](torch.cat(views, 0))
            y = pooled[:m]
            for k in range(1, len(views)):
                y = y + pooled[k * m:(k + 1) * m]
            y = self.post[kind](y)
            for name, (_, std, mean, lo, hi) in self.table[kind].items():
                d = self.out[name](y)
                if self.tanh_output > 0.0:
                    d = self.tanh_output * torch.tanh(d)
                params[name] = _clamp_st(d * std + mean, lo, hi)
        return params


class BondChargeIncrements(nn.Module):
    """Charges: the class-averaged formal charge plus antisymmetric increments along each bond."""

    def __init__(self, node_dim: int, edge_dim: int, pre, out, bound: float, activation: str):
        super().__init__()
        self.bound = float(bound)
        self.pre = _mlp(2 * node_dim + edge_dim, pre[0], pre[1], pre[2], activation)
        self.out = _mlp(pre[1], out[0], 1, out[1], "tanh", bias=False)

    def forward(self, x: Tensor, e: Tensor, bonds: Tensor, bond_edges: Tensor, formal: Tensor, atom_class: Tensor):
        i, j, b = bonds[:, 0], bonds[:, 1], bond_edges
        m = i.shape[0]
        both = self.pre(torch.cat([torch.cat([x[i], e[b], x[j]], -1), torch.cat([x[j], e[b], x[i]], -1)], 0))
        inc = self.bound * torch.tanh(self.out(both[:m] - both[m:]).squeeze(-1))
        q = class_mean(formal.to(inc.dtype).unsqueeze(-1), atom_class).squeeze(-1)
        return q + scatter_sum(inc, i, q.shape[0]) - scatter_sum(inc, j, q.shape[0])


class LennardJonesChargeHead(nn.Module):
    def __init__(self, node_dim: int, edge_dim: int, pre=(512, 512, 4), out=(256, 3), tanh_output: float = 20.0,
                 activation: str = "gelu"):
        super().__init__()
        self.t = float(tanh_output)
        self.sigma = _mlp(node_dim, out[0], 1, out[1], activation)
        self.epsilon = _mlp(node_dim, out[0], 1, out[1], activation)
        self.charge = BondChargeIncrements(node_dim, edge_dim, pre, out, tanh_output, activation)

    def forward(self, x: Tensor, e: Tensor, g: dict) -> Dict[str, Tensor]:
        return {"charge": self.charge(x, e, g["bonds"], g["bond_edges"], g["formal"], g["atom_class"]),
                "sigma": self.t * torch.tanh(self.sigma(x).squeeze(-1)) + self.t,
                "epsilon": self.t * torch.tanh(self.epsilon(x).squeeze(-1)) + self.t}


class Member(nn.Module):
    def __init__(self, graph: dict, bonded: dict, nonbonded: dict, head=None):
        super().__init__()
        self.graph = MolecularGraphTransformer(**graph)
        nd, ed = self.graph.node_dim, self.graph.edge_dim
        self.bonded = BondedHead(nd, ed, **bonded)
        self.nonbonded = (head or LennardJonesChargeHead)(nd, ed, **nonbonded)

    def forward(self, g: dict) -> Dict[str, Tensor]:
        x, e = self.graph(g["features"], g["edge_features"], g["edge_index"], g["atom_class"], g["edge_class"])
        out = self.bonded(x, e, g["terms"])
        out.update(self.nonbonded(x, e, g))
        return out


def split_molecules(n: int, bonds: Sequence[Sequence[int]]) -> List[List[int]]:
    """Connected components (atoms ascending) in order of their first atom."""
    parent = list(range(n))

    def root(a):
        while parent[a] != a:
            parent[a] = parent[parent[a]]
            a = parent[a]
        return a
    for i, j in bonds:
        ri, rj = root(int(i)), root(int(j))
        if ri != rj:
            parent[max(ri, rj)] = min(ri, rj)
    groups: dict = {}
    for a in range(n):
        groups.setdefault(root(a), []).append(a)
    return [groups[r] for r in sorted(groups)]


def _torsion_cos(b1: Tensor, b2: Tensor, b3: Tensor) -> Tensor:
    n1, n2 = torch.linalg.cross(b1, b2, dim=-1), torch.linalg.cross(b2, b3, dim=-1)
    return (n1 * n2).sum(-1) / (n1.norm(dim=-1) * n2.norm(dim=-1))


def _fourier(c: Tensor, k: Tensor) -> Tensor:
    """``sum_n k_n [1 + s_n cos(n phi)]`` for ``n = 1..4``, ``s = (+1, -1, +1, -1)``; ``cos(n phi)``
    by the Chebyshev recursion."""
    c2 = 2.0 * c * c - 1.0
    c3 = 2.0 * c * c2 - c
    c4 = 2.0 * c * c3 - c2
    return k[:, 0] * (1.0 + c) + k[:, 1] * (1.0 - c2) + k[:, 2] * (1.0 + c3) + k[:, 3] * (1.0 - c4)


@register_model("byteff")
class ByteFF(InteratomicPotential):
    """Graph-parameterised classical force field bound to one system (any number of molecules).

    ``graphs`` / ``species``: the distinct :class:`MolecularGraph` objects and, per molecule of the
    system, ``(graph index, atom indices)`` (the system's atom order may interleave molecules). Or
    call :meth:`bind` with the system's atomic numbers and bonds."""

    #: the nonbonded head of every member and its default options
    head = LennardJonesChargeHead
    nonbonded_defaults = dict(pre=(512, 512, 4), out=(256, 3), tanh_output=20.0)

    def __init__(self, graphs: Optional[Sequence[MolecularGraph]] = None, species=None, *, graph: Optional[dict] = None,
                 bonded: Optional[dict] = None, nonbonded: Optional[dict] = None, members: int = 1,
                 supported_elements: Sequence[int] = (1, 6, 7, 8, 9, 15, 16, 17, 35, 53),
                 cutoff: Optional[float] = None, switch_width: float = 0.0, coulomb_constant: float = COULOMB,
                 fudge_qq: float = 0.8333333333, fudge_lj: float = 0.5, reference_positions=None):
        super().__init__()
        self.graph_options = {**GRAPH_DEFAULTS, **(graph or {})}
        self.bonded_options = {**dict(pre=(256, 256, 3), out=(256, 4), tanh_output=20.0, form="harmonic"),
                               **(bonded or {})}
        self.nonbonded_options = {**self.nonbonded_defaults, **(nonbonded or {})}
        self.members = nn.ModuleList(Member(self.graph_options, self.bonded_options, self.nonbonded_options,
                                            self.head) for _ in range(int(members)))
        self.supported_elements = tuple(int(z) for z in supported_elements)
        self.coulomb_constant, self.fudge_qq, self.fudge_lj = float(coulomb_constant), float(fudge_qq), float(fudge_lj)
        self.all_pairs = cutoff is None
        self.cutoff = 0.1 if cutoff is None else float(cutoff)
        self.switch_width = float(switch_width)
        if not self.all_pairs and not 0.0 <= self.switch_width < self.cutoff:
            raise ValueError("switch_width must satisfy 0 <= switch_width < cutoff")
        self.node_feature_dim = 1
        self.bound = False
        self._cache = None
        if graphs is not None:
            self.bind_graphs(graphs, species, reference_positions)

    # ------------------------------------------------------------------------------ binding
    def bind(self, atomic_numbers, bonds, bond_orders=None, formal_charges=None, reference_positions=None) -> "ByteFF":
        """Bind a system given by its atoms and bonds: molecules are its connected components, and
        molecules with the same graph (same atoms in the same order) share one prediction."""
        z = [int(v) for v in atomic_numbers]
        bonds = [(int(i), int(j)) for i, j in bonds]
        orders = [1.0] * len(bonds) if bond_orders is None else [float(o) for o in bond_orders]
        fc = [0] * len(z) if formal_charges is None else [int(c) for c in formal_charges]
        graphs, keys, species = [], {}, []
        for atoms in split_molecules(len(z), bonds):
            local = {a: k for k, a in enumerate(atoms)}
            mb = [(local[i], local[j], o) for (i, j), o in zip(bonds, orders) if i in local]
            key = (tuple(z[a] for a in atoms), tuple(fc[a] for a in atoms), tuple(sorted(mb)))
            if key not in keys:
                keys[key] = len(graphs)
                graphs.append(molecular_graph_from_bonds([z[a] for a in atoms], [(i, j) for i, j, _ in mb],
                                                         [o for _, _, o in mb], [fc[a] for a in atoms]))
            species.append((keys[key], atoms))
        return self.bind_graphs(graphs, species, reference_positions)

    def bind_graphs(self, graphs: Sequence[MolecularGraph], species=None, reference_positions=None) -> "ByteFF":
        graphs = list(graphs)
        if species is None:
            species, at = [], 0
            for k, g in enumerate(graphs):
                species.append((k, list(range(at, at + g.n_atoms))))
                at += g.n_atoms
        cat = np.concatenate
        node_off = np.cumsum([0] + [g.n_atoms for g in graphs])
        edge_off = np.cumsum([0] + [2 * g.bonds.shape[0] for g in graphs])
        names = ("bonds", "angles", "propers", "impropers")
        term_off = {k: np.cumsum([0] + [getattr(g, k).shape[0] for g in graphs]) for k in names}
        u = {"features": cat([np.stack([g.atomic_numbers - 1, g.degree, g.formal_charges, g.ring_degree, g.min_ring], 1)
                              for g in graphs]),
             "edge_features": cat([g.edge_features() for g in graphs]),
             "edge_index": cat([g.edge_index() + o for g, o in zip(graphs, node_off)], 1),
             "atom_class": cat([g.atom_class + o for g, o in zip(graphs, node_off)]),
             "edge_class": cat([g.edge_class + o for g, o in zip(graphs, edge_off)]),
             "formal": cat([g.formal_charges for g in graphs]),
             "bonds": cat([g.bonds + o for g, o in zip(graphs, node_off)]).reshape(-1, 2),
             "bond_edges": cat([2 * np.arange(g.bonds.shape[0]) + o for g, o in zip(graphs, edge_off)]),
             "linear": cat([g.proper_linear for g in graphs])}
        u["element"] = u["features"][:, 0]
        dev = next(self.parameters()).device

        def buf(name, value, dtype=torch.long):
            self.register_buffer(name, torch.as_tensor(np.asarray(value), dtype=dtype, device=dev), persistent=False)
        for k, v in u.items():
            buf("_u_" + k, v, torch.bool if k == "linear" else torch.long)
        edge_names = {"bond": None, "angle": "angle_edges", "proper": "proper_edges", "improper": "improper_edges"}
        width = {"bond": 2, "angle": 3, "proper": 4, "improper": 4}
        for kind, name in zip(edge_names, names):
            atoms = cat([getattr(g, name) + o for g, o in zip(graphs, node_off)]).reshape(-1, width[kind])
            ed = (u["bond_edges"].reshape(-1, 1) if kind == "bond"
                  else cat([getattr(g, edge_names[kind]) + o for g, o in zip(graphs, edge_off)])
                  .reshape(-1, 3 if kind == "improper" else width[kind] - 1))
            buf(f"_t_{kind}_atoms", atoms)
            buf(f"_t_{kind}_edges", ed)
        sys_atom, mol_of = [], []
        sys_terms, sys_src = {k: [] for k in names}, {k: [] for k in names}
        sys_pairs = {k: [] for k in ("pairs12", "pairs13", "pairs14", "pairs15")}
        for m, (s, atoms) in enumerate(species):
            g, idx = graphs[s], np.asarray(atoms, dtype=np.int64)
            sys_atom.append(np.arange(g.n_atoms) + node_off[s])
            mol_of.append(np.full(g.n_atoms, m))
            for k in names:
                keep = ~g.proper_linear if k == "propers" else np.ones(getattr(g, k).shape[0], dtype=bool)
                sys_terms[k].append(idx[getattr(g, k)][keep].reshape(-1, width[k[:-1]]))
                sys_src[k].append((np.arange(getattr(g, k).shape[0]) + term_off[k][s])[keep])
            for k in sys_pairs:
                sys_pairs[k].append(idx[getattr(g, k)].reshape(-1, 2))
        order = np.argsort(cat([np.asarray(a) for _, a in species]))
        n = order.shape[0]
        if not np.array_equal(np.sort(cat([np.asarray(a) for _, a in species])), np.arange(n)):
            raise ValueError("the molecules' atom indices must cover 0 .. n-1 once each")
        self.n_atoms = n
        buf("_atom_src", cat(sys_atom)[order])
        buf("_z", (u["features"][:, 0] + 1)[cat(sys_atom)][order])
        for k in names:
            buf(f"_{k}", cat(sys_terms[k]).T)
            buf(f"_{k}_src", cat(sys_src[k]))
        for k, v in sys_pairs.items():
            buf("_" + k, cat(v).T)
        buf("_molecule", cat(mol_of)[order])
        self._bind_pairs(n)
        self._bind_hypervalent(graphs, species, reference_positions)
        self.species = sorted({int(z) for z in self._z.tolist()})
        self.bound = True
        self._cache = None
        return self

    def _bind_pairs(self, n: int) -> None:
        self.register_buffer("_excluded", torch.cat([self._pairs12, self._pairs13, self._pairs14], 1), persistent=False)
        pairs = self._pairs14
        if self.all_pairs:
            i, j = torch.triu_indices(n, n, 1, device=pairs.device)
            code = torch.zeros(n, n, dtype=torch.int8, device=pairs.device)
            for c, pp in ((1, self._pairs12), (1, self._pairs13), (2, self._pairs14)):
                code[pp[0], pp[1]] = c
            far = code[i, j] == 0
            pairs = torch.cat([pairs, torch.stack([i[far], j[far]])], 1)
        self.register_buffer("_pair_list", pairs, persistent=False)
        self._plans = {}

    def _bind_hypervalent(self, graphs, species, positions) -> None:
        hyper = torch.as_tensor(np.concatenate([g.hypervalent for g in graphs]), device=self._u_features.device)
        masks = {"bond": hyper[self._t_bond_atoms].any(1), "angle": hyper[self._t_angle_atoms[:, 1]],
                 "proper": hyper[self._t_proper_atoms].any(1), "improper": hyper[self._t_improper_atoms].any(1)}
        for kind, m in masks.items():
            self.register_buffer(f"_t_{kind}_hyper", m, persistent=False)
        ref = {k: torch.full((int(masks[k].shape[0]),), float("nan"), dtype=torch.float64) for k in ("bond", "angle")}
        if bool(hyper.any()) and positions is not None:
            pos = np.asarray(positions, dtype=np.float64).reshape(-1, 3)
            node_off = np.cumsum([0] + [g.n_atoms for g in graphs])
            to_global, seen = np.zeros(int(node_off[-1]), dtype=np.int64), set()
            for s, atoms in species:
                if s not in seen:
                    seen.add(s)
                    to_global[node_off[s]:node_off[s + 1]] = atoms
            x = torch.as_tensor(pos[to_global])
            b, a = self._t_bond_atoms.cpu(), self._t_angle_atoms.cpu()
            ref["bond"] = torch.linalg.norm(x[b[:, 1]] - x[b[:, 0]], dim=1)
            u, v = x[a[:, 0]] - x[a[:, 1]], x[a[:, 2]] - x[a[:, 1]]
            ref["angle"] = torch.atan2(torch.linalg.cross(u, v, dim=-1).norm(dim=-1), (u * v).sum(-1))
        elif bool(hyper.any()):
            import warnings
            warnings.warn("hypervalent P/S centres: their bonds and angles have no predicted equilibrium values; "
                          "pass reference_positions (an optimised geometry) when binding", stacklevel=3)
        for k, v in ref.items():
            v = torch.where(masks[k].cpu(), v, torch.full_like(v, float("nan")))
            self.register_buffer(f"_t_{k}_x0", v.to(self._u_features.device), persistent=False)

    @property
    def atomic_numbers(self) -> Tensor:
        return self._z

    def term_atoms(self, kind: str) -> Tensor:
        """``(M, k)`` atoms of each distinct term (``bond``, ``angle``, ``proper``, ``improper``) in
        the unique-graph numbering that :meth:`predicted_parameters` follows."""
        return getattr(self, f"_t_{kind}_atoms")

    # ---------------------------------------------------------------------------- parameters
    def _unique_graph(self) -> dict:
        g = {k: getattr(self, "_u_" + k) for k in ("features", "edge_features", "edge_index", "atom_class",
                                                  "edge_class", "formal", "bonds", "bond_edges", "element")}
        g["terms"] = {k: (getattr(self, f"_t_{k}_atoms"), getattr(self, f"_t_{k}_edges")) for k in TERM_ATOMS}
        return g

    def _patch(self, p: dict) -> dict:
        out = dict(p)
        for kind, k_fixed in HYPERVALENT_K.items():
            m = getattr(self, f"_t_{kind}_hyper").unsqueeze(-1)
            for name in (f"{kind}_k", f"{kind}_k1"):
                if name in out:
                    out[name] = torch.where(m, torch.full_like(out[name], k_fixed), out[name])
            for name in (f"{kind}_r0" if kind == "bond" else "angle_d0", f"{kind}_k2"):
                if name in out:
                    out[name] = torch.where(m, torch.zeros_like(out[name]), out[name])
        for kind in ("proper", "improper"):
            m = getattr(self, f"_t_{kind}_hyper").unsqueeze(-1)
            out[f"{kind}_k"] = torch.where(m, torch.zeros_like(out[f"{kind}_k"]), out[f"{kind}_k"])
        return out

    def _derive(self, p: dict) -> dict:
        out = {k: v for k, v in p.items() if not k.startswith(("bond_", "angle_"))}
        if "bond_k1" in p:
            for kind, (b1, b2) in (("bond", TWO_WELL_BONDS), ("angle", TWO_WELL_ANGLES)):
                k1, k2 = p[f"{kind}_k1"].squeeze(-1), p[f"{kind}_k2"].squeeze(-1)
                out[f"{kind}_k"], out[f"{kind}_x0"] = k1 + k2, (k1 * b1 + k2 * b2) / (k1 + k2)
        else:
            out["bond_k"], out["bond_x0"] = p["bond_k"].squeeze(-1), p["bond_r0"].squeeze(-1)
            out["angle_k"], out["angle_x0"] = p["angle_k"].squeeze(-1), torch.deg2rad(p["angle_d0"].squeeze(-1))
        for kind in ("bond", "angle"):
            ref = getattr(self, f"_t_{kind}_x0").to(out[f"{kind}_x0"].dtype)
            out[f"{kind}_x0"] = torch.where(torch.isnan(ref), out[f"{kind}_x0"], ref)
        out["proper_k"] = p["proper_k"] * (~self._u_linear).to(p["proper_k"].dtype).unsqueeze(-1)
        return out

    def predicted_parameters(self, per_member: bool = False) -> Dict[str, Tensor]:
        """The ensemble-mean parameters per distinct atom / term (kcal/mol, Angstrom, radians):
        ``bond_k``, ``bond_x0``, ``angle_k``, ``angle_x0``, ``proper_k`` (``(M, 4)``), ``improper_k``,
        ``charge``, ``sigma``, ``epsilon`` (``per_member``: each member's raw outputs stacked)."""
        if not self.bound:
            raise RuntimeError("bind a system first (model.bind(...))")
        g = self._unique_graph()
        outs = [self._patch(m(g)) for m in self.members]
        if per_member:
            return {k: torch.stack([o[k] for o in outs]) for k in outs[0]}
        return self._derive({k: torch.stack([o[k] for o in outs]).mean(0) for k in outs[0]})

    def _params_cached(self) -> Dict[str, Tensor]:
        """Predicted once per weight version outside training (the graph network is independent of
        the coordinates); recomputed every call while training."""
        if self.training:
            return self.predicted_parameters()
        params = tuple(self.parameters())
        key = (tuple(p._version for p in params), tuple(p.data_ptr() for p in params), params[0].dtype,
               params[0].device)
        if self._cache is None or self._cache[0] != key:
            with torch.no_grad():
                self._cache = (key, self.predicted_parameters())
        return self._cache[1]

    # ------------------------------------------------------------------------------- energy
    def _check(self, data: AtomicGraph) -> int:
        if not self.bound:
            raise RuntimeError("bind a system first (model.bind(...))")
        n, B = self.n_atoms, data.num_graphs
        if not bool((data.n_atoms == n).all()):
            raise ValueError(f"every structure must have the bound system's {n} atoms (got {data.n_atoms.tolist()})")
        if not bool((data.atomic_numbers.view(B, n) == self._z).all()):
            raise ValueError("atomic numbers do not match the bound system's element sequence")
        if not self.training and self.supported_elements:
            bad = sorted(set(self.species) - set(self.supported_elements))
            if bad:
                raise ValueError(f"elements {bad} are not supported by this model "
                                 f"(supported: {list(self.supported_elements)})")
        if self.all_pairs and data.cell is not None:
            raise ValueError("this model evaluates every pair of a structure and takes no cell; "
                             "set a cutoff for periodic systems")
        return B

    def _plan(self, B: int, device) -> dict:
        key = (B, str(device))
        if key not in self._plans:
            off = torch.arange(B, device=device) * self.n_atoms

            def ex(idx: Tensor) -> Tensor:
                return (idx.unsqueeze(1) + off.view(1, B, 1)).reshape(idx.shape[0], -1)
            n14 = self._pairs14.shape[1]
            self._plans[key] = {"bonds": ex(self._bonds), "angles": ex(self._angles), "propers": ex(self._propers),
                                "impropers": ex(self._impropers), "pairs": ex(self._pair_list),
                                "is14": (torch.arange(self._pair_list.shape[1], device=device) < n14).repeat(B)}
        return self._plans[key]

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        B = self._check(data)
        N = data.num_nodes
        plan = self._plan(B, data.pos.device)
        dt = data.model_dtype
        P = {k: v.to(dt) for k, v in self._params_cached().items()}
        atom = {k: P[k][self._atom_src].repeat(B) for k in ("charge", "sigma", "epsilon")}
        b, a, tp, ti, pr = (plan[k] for k in ("bonds", "angles", "propers", "impropers", "pairs"))
        # bonds and angles
        vb = pair_vectors(data, b[0], b[1])
        e_bond = 0.5 * P["bond_k"][self._bonds_src].repeat(B) * (vb.norm(dim=1) - P["bond_x0"][self._bonds_src].repeat(B)) ** 2
        u, v = pair_vectors(data, a[1], a[0]), pair_vectors(data, a[1], a[2])
        theta = torch.atan2(torch.linalg.cross(u, v, dim=-1).norm(dim=-1), (u * v).sum(-1))
        e_angle = 0.5 * P["angle_k"][self._angles_src].repeat(B) * (theta - P["angle_x0"][self._angles_src].repeat(B)) ** 2

        def torsion_cos(t):
            return _torsion_cos(pair_vectors(data, t[0], t[1]), pair_vectors(data, t[1], t[2]),
                                pair_vectors(data, t[2], t[3]))
        e_tors = _fourier(torsion_cos(tp), P["proper_k"][self._propers_src].repeat(B, 1))
        e_impr = P["improper_k"][self._impropers_src].repeat(B, 1)[:, 0] * (1.0 - (2.0 * torsion_cos(ti) ** 2 - 1.0))
        # listed pairs: the 1-4 pairs (scaled), and all other non-excluded pairs without a cutoff
        is14 = plan["is14"]
        q, sig, eps = atom["charge"], atom["sigma"], atom["epsilon"]
        vp = pair_vectors(data, pr[0], pr[1])
        r2 = (vp * vp).sum(1)
        lj_s = torch.where(is14, torch.full_like(r2, self.fudge_lj), torch.ones_like(r2))
        qq_s = torch.where(is14, torch.full_like(r2, self.fudge_qq), torch.ones_like(r2))
        sigma = 0.5 * (sig[pr[0]] + sig[pr[1]])
        x = (sigma * sigma / r2) ** 3
        vdw = 4.0 * lj_s * geometric_mean(eps[pr[0]], eps[pr[1]]) * (x * x - x)
        coul = self.coulomb_constant * qq_s * q[pr[0]] * q[pr[1]] / torch.sqrt(r2)

        def halves(e, i, j, mask=None):
            e = e if mask is None else e * mask.to(e.dtype)
            return scatter_sum(0.5 * e, i, N) + scatter_sum(0.5 * e, j, N)
        m14, far = is14, ~is14
        node = {"e_bond": halves(e_bond, b[0], b[1]), "e_angle": scatter_sum(e_angle, a[1], N),
                "e_torsion": scatter_sum(e_tors, tp[1], N), "e_improper": scatter_sum(e_impr, ti[0], N),
                "e_vdw": halves(vdw, pr[0], pr[1], far), "e_coulomb": halves(coul, pr[0], pr[1], far),
                "e_vdw14": halves(vdw, pr[0], pr[1], m14), "e_coulomb14": halves(coul, pr[0], pr[1], m14)}
        if not self.all_pairs:
            src, dst, vec, r2n, half, included = half_edges(data, self._excluded, self.n_atoms,
                                                            self.__dict__.setdefault("_exclusion_keys", {}))
            r = torch.sqrt(r2n)
            w = included.to(r.dtype) * half * quintic_switch(r, self.cutoff, self.switch_width)
            s = 0.5 * (sig[src] + sig[dst])
            xn = (s * s / r2n) ** 3
            node["e_vdw"] = node["e_vdw"] + halves(w * 4.0 * geometric_mean(eps[src], eps[dst]) * (xn * xn - xn),
                                                   src, dst)
            node["e_coulomb"] = node["e_coulomb"] + halves(w * self.coulomb_constant * q[src] * q[dst] / r, src, dst)
        total = sum(node.values()) * KCAL_TO_EV
        out = {"node_energy": total, "energy": self.aggregate_energy(total, data)}
        out.update({k: v.view(B, -1).to(torch.float64).sum(1) * KCAL_TO_EV for k, v in node.items()})
        out["charges"] = q
        out["node_features"] = q.unsqueeze(1)
        return out

    @classmethod
    def from_config(cls, cfg) -> "ByteFF":
        e = dict(cfg.extra or {})
        kw = {k: e[k] for k in ("graph", "bonded", "nonbonded", "members", "supported_elements", "switch_width",
                                "coulomb_constant", "fudge_qq", "fudge_lj") if e.get(k) is not None}
        kw["cutoff"] = None if e.get("all_pairs", True) else float(cfg.cutoff)
        model = cls(**kw)
        if e.get("atomic_numbers") is not None and e.get("bonds") is not None:
            model.bind(e["atomic_numbers"], e["bonds"], e.get("bond_orders"), e.get("formal_charges"))
        return model
