"""High-dimensional neural network potentials, generations 1 to 4 (Behler, Chem. Rev. 121,
10037, 2021), in the conventions of the RuNNer code as the reference has them
(``src/xnn/dnn/models/hdnnp.py:168-841``):

* 1G (:class:`NNP1G`): one network on the ``n (n-1) / 2`` distances (or ``1/r``,
  ``exp(-r/l)``) of a fixed system, optionally averaged over permutations of like atoms;
* 2G: per-element networks on atom-centred symmetry functions;
* 3G: a second set of element networks gives charges (shifted uniformly to the net charge) whose
  Gaussian-charge electrostatics add to the energy;
* 4G: the networks give electronegativities; charges follow from a charge equilibration with
  Gaussian charges and element hardnesses (constants ``J = act(p_Z)`` or networks) over the whole
  structure (Ewald-summed in a cell), and enter the short-range networks as ``(q - c_Z) s_Z``.

Gaussian widths default to ``0.45 r_cov`` clamped to ``[0.25, 0.6]`` A; an optional screening
cutoff removes the electrostatics inside the short-range sphere.
"""
from __future__ import annotations

import itertools
import math
from typing import Iterable, Optional, Sequence

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..data.elements import ATOMIC_NUMBERS
from ..featurizers.acsf import AtomCenteredSymmetryFunctions, cutoff_function
from ..nn.blocks import make_activation
from ..ops.scatter import scatter_sum
from .base import InteratomicPotential
from .charges import gaussian_coulomb_matrix, solve_charges
from .descriptor import DescriptorPotential, ElementNetworks
from .electrostatics import COULOMB_CONSTANT
from .registry import register_model

# covalent radii in A (WebElements) by atomic number; None where none is tabulated
COVALENT_RADII = (
    None, 0.37, 0.32, 1.34, 0.90, 0.82, 0.77, 0.75, 0.73, 0.71, 0.69, 1.54, 1.30, 1.18, 1.11, 1.06, 1.02, 0.99, 0.97,
    1.96, 1.74, 1.44, 1.36, 1.25, 1.27, 1.39, 1.25, 1.26, 1.21, 1.38, 1.31, 1.26, 1.22, 1.19, 1.16, 1.14, 1.10,
    2.11, 1.92, 1.62, 1.48, 1.37, 1.45, 1.56, 1.26, 1.35, 1.31, 1.53, 1.48, 1.44, 1.41, 1.38, 1.35, 1.33, 1.30,
    2.25, 1.98, 1.69, None, None, None, None, None, None, None, None, None, None, None, None, None, 1.60, 1.50, 1.38,
    1.46, 1.59, 1.28, 1.37, 1.28, 1.44, 1.49, 1.48, 1.47, 1.46, None, None, 1.45)


def _z(v) -> int:
    return ATOMIC_NUMBERS[v] if isinstance(v, str) and not v.isdigit() else int(v)


def default_gaussian_widths(species: Sequence[int]) -> list:
    out = []
    for z in species:
        r = COVALENT_RADII[z] if z < len(COVALENT_RADII) else None
        if r is None:
            raise ValueError(f"no covalent radius for Z={z}; give gaussian_widths explicitly")
        out.append(min(0.6, max(0.25, 0.45 * r)))
    return out


def default_symmetry_functions(species: Sequence[int], cutoff: float, n_radial: int = 6, angular: bool = True):
    """Radial type-2 functions ``eta = (m / r_c)^2`` (``m = 1..n_radial``) per element pair and angular
    type-3 functions (``eta = 1 / r_c^2``, ``lambda = +-1``, ``zeta = 1, 4``) per neighbour pair."""
    funcs = []
    for zc in species:
        for zn in species:
            for m in range(1, n_radial + 1):
                funcs.append({"element": zc, "type": 2, "neighbors": [zn], "eta": (m / cutoff) ** 2, "rs": 0.0})
        if angular:
            for za, zb in itertools.combinations_with_replacement(species, 2):
                for zeta in (1.0, 4.0):
                    for lam in (-1.0, 1.0):
                        funcs.append({"element": zc, "type": 3, "neighbors": [za, zb], "eta": 1.0 / cutoff ** 2,
                                      "lambda": lam, "zeta": zeta})
    return [{"kind": "cosine", "r_cut": float(cutoff)}], funcs


def _per_species(value, species, name):
    if isinstance(value, dict):
        table = {_z(k): float(v) for k, v in value.items()}
        missing = [z for z in species if z not in table]
        if missing:
            raise ValueError(f"{name}: no value for elements {missing}")
        return [table[z] for z in species]
    vals = [float(v) for v in value]
    if len(vals) != len(species):
        raise ValueError(f"{name}: {len(vals)} values for {len(species)} species")
    return vals


@register_model("hdnnp")
class HDNNP(DescriptorPotential):
    head_modules = ("element_nets", "_self_energies_by_z")

    def __init__(self, species: Sequence[int], featurizer: AtomCenteredSymmetryFunctions, generation: int = 2,
                 hidden=(15, 15), activation="tanh", atomic_energies=None, charge_featurizer=None, charge_hidden=None,
                 charge_activation=None, constrain_charges: bool = True, gaussian_widths=None,
                 screening: Optional[dict] = None, hardness: str = "element", hardness_init=10.0,
                 hardness_activation: str = "linear", hardness_hidden=None, hardness_activation_nn=None,
                 charge_neuron: bool = True, ewald_accuracy: float = 1e-10,
                 coulomb_constant: float = COULOMB_CONSTANT, energy_scale: float = 1.0, chi_scale: float = 1.0,
                 hardness_scale: float = 1.0):
        if generation not in (2, 3, 4):
            raise ValueError(f"HDNNP generation must be 2, 3 or 4 (1: NNP1G), got {generation}")
        species = [int(z) for z in species]
        extra = 1 if generation == 4 and charge_neuron else 0
        super().__init__(featurizer, species, hidden, activation, True, atomic_energies, extra)
        self.generation = int(generation)
        self.charge_neuron = bool(extra)
        self.register_buffer("energy_scale", torch.tensor(float(energy_scale)))
        self.charge_featurizer = charge_featurizer
        self.charge_nets = self.hardness_nets = self.hardness_raw = None
        self.hardness = hardness
        self.constrain_charges = bool(constrain_charges)
        self.screening = None if screening is None else dict(screening)
        self.ewald_accuracy = float(ewald_accuracy)
        self.coulomb_constant = float(coulomb_constant)
        gen4 = generation == 4
        if gen4 and hardness not in ("element", "network"):
            raise ValueError(f"hardness must be 'element' or 'network', got {hardness!r}")
        # buffers by generation: name -> (value, saved in the state dict); the ones a generation
        # does not use exist as inert defaults outside the state dict
        q_feat = charge_featurizer if charge_featurizer is not None else featurizer
        q_dims = getattr(q_feat, "n_features", None) or q_feat.output_dim
        sigma = torch.zeros(119)
        if generation >= 3:
            widths = (default_gaussian_widths(species) if gaussian_widths is None
                      else _per_species(gaussian_widths, species, "gaussian_widths"))
            sigma[torch.tensor(species)] = torch.tensor(widths, dtype=sigma.dtype)
        slot = torch.zeros(119, dtype=torch.long)
        if gen4 and hardness == "element":
            slot.fill_(-1)
            slot[torch.tensor(species)] = torch.arange(len(species))
        buffers = {
            "gaussian_widths": (sigma, generation >= 3),
            "chi_scale": (torch.tensor(float(chi_scale) if gen4 else 1.0), gen4),
            "hardness_scale": (torch.tensor(float(hardness_scale) if gen4 else 1.0), gen4),
            "charge_input_shift": (torch.zeros(119), gen4),
            "charge_input_factor": (torch.ones(119), gen4),
            "_hardness_index": (slot, False),
        }
        for name, (value, saved) in buffers.items():
            self.register_buffer(name, value, persistent=saved)
        self.hardness_act = nn.Identity()
        if generation >= 3:
            self.charge_nets = ElementNetworks(species, q_dims, hidden if charge_hidden is None else charge_hidden,
                                               activation if charge_activation is None else charge_activation)
            self.cutoff = max(self.cutoff, q_feat.cutoff, float(self.screening["r_cut"]) if self.screening else 0.0)
        if gen4 and hardness == "element":
            init = ([float(hardness_init)] * len(species) if isinstance(hardness_init, (int, float))
                    else _per_species(hardness_init, species, "hardness_init"))
            self.hardness_raw = nn.Parameter(torch.tensor(init))
            self.hardness_act = make_activation(hardness_activation)
        elif gen4:
            self.hardness_nets = ElementNetworks(
                species, q_dims, hidden if hardness_hidden is None else hardness_hidden,
                activation if hardness_activation_nn is None else hardness_activation_nn)

    # ------------------------------------------------------------------ electrostatics
    def coulomb_matrices(self, data: AtomicGraph, dtype) -> list:
        z, pos, out = data.atomic_numbers, data.pos.to(dtype), []
        for b in range(data.num_graphs):
            idx = (data.batch == b).nonzero().flatten()
            cell = None
            if data.cell is not None and data.pbc is not None and bool(data.pbc[b].any()):
                if not bool(data.pbc[b].all()):
                    raise NotImplementedError("HDNNP electrostatics need full or no periodicity")
                cell = data.cell[b].to(dtype)
            a = gaussian_coulomb_matrix(pos[idx], self.gaussian_widths.to(dtype)[z[idx]], cell, self.ewald_accuracy)
            out.append((idx, self.coulomb_constant * a))
        return out

    def charges_and_parameters(self, data: AtomicGraph, desc: Tensor, desc_q: Tensor, matrices=None) -> dict:
        z = data.atomic_numbers
        total = data.total_charge.to(desc.dtype) if data.total_charge is not None else desc.new_zeros(data.num_graphs)
        if self.generation == 3:
            raw = self.charge_nets(desc_q, z)
            excess = (scatter_sum(raw, data.batch, data.num_graphs) - total) / data.n_atoms.to(raw.dtype)
            return {"charges_raw": raw, "charges": raw - excess[data.batch] if self.constrain_charges else raw}
        chi = self.chi_scale.to(desc.dtype) * self.charge_nets(desc_q, z)
        hard = (self.hardness_nets(desc_q, z) if self.hardness_nets is not None
                else self.hardness_act(self.hardness_raw.to(desc.dtype))[self._hardness_index[z]])
        hard = self.hardness_scale.to(desc.dtype) * hard
        matrices = self.coulomb_matrices(data, desc.dtype) if matrices is None else matrices
        q, mus = torch.zeros_like(chi), []
        for b, (idx, a) in enumerate(matrices):
            qb, mub = solve_charges(chi[idx], hard[idx], a, total[b])
            q = q.index_put((idx,), qb)
            mus.append(mub)
        return {"charges": q, "electronegativities": chi, "hardness": hard, "chemical_potential": torch.cat(mus)}

    def electrostatic_energy(self, data: AtomicGraph, charges: Tensor, matrices=None) -> Tensor:
        matrices = self.coulomb_matrices(data, charges.dtype) if matrices is None else matrices
        node = torch.zeros_like(charges)
        for idx, a in matrices:
            qb = charges[idx]
            node = node.index_put((idx,), 0.5 * qb * (a @ qb))
        if self.screening is not None:
            node = node - self.coulomb_constant * self._screening_terms(data.atomic_numbers, data.edge_index,
                                                                        data.edge_vectors(), charges)
        return node

    def _screening_terms(self, z: Tensor, edge_index: Tensor, edge_vec: Tensor, q: Tensor) -> Tensor:
        s = self.screening
        r = torch.linalg.norm(edge_vec.to(q.dtype), dim=-1)
        src, dst = edge_index[0], edge_index[1]
        fc = cutoff_function(r, str(s.get("kind", "cosine")), float(s["r_cut"]), float(s.get("r_inner", 0.0) or 0.0),
                             int(s.get("exponent", 2)))
        sigma = self.gaussian_widths.to(q.dtype)[z]
        g2 = sigma[src] ** 2 + sigma[dst] ** 2
        point = g2 <= 0
        kern = torch.where(point, torch.ones_like(r),
                           torch.special.erf(r / torch.sqrt(2.0 * torch.where(point, torch.ones_like(g2), g2)))) / r
        node = scatter_sum(0.5 * q[dst] * q[src] * kern * fc, dst, q.shape[0])
        return node + torch.where(sigma > 0, q * q / (2.0 * math.sqrt(math.pi) * torch.where(
            sigma > 0, sigma, torch.ones_like(sigma))), torch.zeros_like(q))

    def charge_input(self, data: AtomicGraph, charges: Tensor) -> Tensor:
        z = data.atomic_numbers
        return (charges - self.charge_input_shift.to(charges.dtype)[z]) * self.charge_input_factor.to(charges.dtype)[z]

    # ------------------------------------------------------------------ evaluation
    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        if self.generation >= 3:
            raise RuntimeError("3G and 4G HDNNP models need the whole structure (global charges)")
        desc = self.featurizer.compute(atomic_numbers, edge_index, edge_vec, atomic_numbers.shape[0])
        short = self.energy_scale.to(desc.dtype) * self.element_nets(desc, atomic_numbers)
        return desc, short + self._self_energies_by_z.to(desc.dtype)[atomic_numbers]

    def forward(self, data: AtomicGraph) -> dict:
        desc = self.featurizer(data)
        z = data.atomic_numbers
        out, extra, matrices = {}, None, None
        if self.generation >= 3:
            desc_q = desc if self.charge_featurizer is None else self.charge_featurizer(data)
            matrices = self.coulomb_matrices(data, desc.dtype)
            out.update(self.charges_and_parameters(data, desc, desc_q, matrices))
            if self.charge_neuron:
                extra = self.charge_input(data, out["charges"])[:, None]
        short = self.energy_scale.to(desc.dtype) * self.element_nets(desc, z, extra) + \
            self._self_energies_by_z.to(desc.dtype)[z]
        node = short
        out["node_energy_short"] = short
        out["energy_short"] = self.aggregate_energy(short, data)
        if self.generation >= 3:
            elec = self.electrostatic_energy(data, out["charges"], matrices)
            node = node + elec
            out["energy_elec"] = self.aggregate_energy(elec, data)
            if data.cell is None:
                out["dipole"] = scatter_sum(out["charges"][:, None] * data.pos.to(desc.dtype), data.batch,
                                            data.num_graphs)
        out["node_energy"] = node
        out["energy"] = self.aggregate_energy(node, data)
        out["node_features"] = desc
        return out

    @torch.no_grad()
    def fit_scaling(self, graphs: Iterable[AtomicGraph], mode: Optional[str] = None,
                    charge_mode: Optional[str] = None) -> None:
        graphs = list(graphs)
        self.featurizer.fit_scaling(graphs, mode)
        if self.charge_featurizer is not None:
            self.charge_featurizer.fit_scaling(graphs, charge_mode or mode)

    @classmethod
    def from_config(cls, cfg):
        e = dict(cfg.extra or {})
        generation = int(e.get("generation", 2))
        if generation == 1:
            return NNP1G.from_config(cfg)
        species = [_z(z) for z in e.get("species", [1, 6, 8])]
        cutoffs, functions = e.get("cutoffs"), e.get("symmetry_functions")
        if functions is None:
            if "etas" in e or "rs" in e:
                cutoffs = [{"kind": "cosine", "r_cut": float(cfg.cutoff)}]
                functions = [{"element": zc, "type": 2, "neighbors": [zn], "eta": float(eta), "rs": float(rs)}
                             for zc in species for zn in species for eta in e.get("etas", (0.05, 0.5, 2.0, 8.0))
                             for rs in e.get("rs", (0.0,))]
            else:
                cutoffs, functions = default_symmetry_functions(species, float(cfg.cutoff))
        feat = AtomCenteredSymmetryFunctions(species, cutoffs, functions, mode=e.get("scaling", "none"),
                                             scale_range=e.get("scale_range", (0.0, 1.0)))
        cfeat = None
        if e.get("charge_symmetry_functions") is not None:
            cfeat = AtomCenteredSymmetryFunctions(species, e.get("charge_cutoffs", cutoffs),
                                                  e["charge_symmetry_functions"],
                                                  mode=e.get("charge_scaling", e.get("scaling", "none")),
                                                  scale_range=e.get("scale_range", (0.0, 1.0)))
        ae = e.get("atomic_energies")
        model = cls(species, feat, generation=generation, hidden=e.get("hidden", (15, 15)),
                    activation=e.get("activation", "tanh"),
                    atomic_energies=None if ae is None else _per_species(ae, species, "atomic_energies"),
                    charge_featurizer=cfeat, charge_hidden=e.get("charge_hidden"),
                    charge_activation=e.get("charge_activation"), gaussian_widths=e.get("gaussian_widths"),
                    screening=e.get("screening"), hardness=e.get("hardness", "element"),
                    hardness_init=e.get("hardness_init", 10.0),
                    hardness_activation=e.get("hardness_activation", "linear"),
                    hardness_hidden=e.get("hardness_hidden"), charge_neuron=bool(e.get("charge_neuron", True)),
                    constrain_charges=bool(e.get("constrain_charges", True)),
                    ewald_accuracy=float(e.get("ewald_accuracy", 1e-10)))
        if model.cutoff > float(cfg.cutoff) + 1e-9:
            raise ValueError(f"the symmetry functions (or screening) reach {model.cutoff:g}, beyond the config "
                             f"cutoff {float(cfg.cutoff):g}; raise model.cutoff")
        return model


def like_atom_permutations(species: Sequence[int], limit: int) -> list:
    """Every permutation of atom indices that only exchanges atoms of one element."""
    groups: dict = {}
    for i, z in enumerate(species):
        groups.setdefault(int(z), []).append(i)
    size = 1
    for members in groups.values():
        size *= math.factorial(len(members))
    if size > limit:
        raise ValueError(f"symmetrizing over {size} permutations exceeds max_permutations={limit}")
    perms = [list(range(len(species)))]
    for members in groups.values():
        grown = []
        for base in perms:
            for order in itertools.permutations(members):
                p = list(base)
                for s, d in zip(members, order):
                    p[s] = d
                grown.append(p)
        perms = grown
    return perms


@register_model("nnp1g")
class NNP1G(InteratomicPotential):
    def __init__(self, species: Sequence[int], hidden=(30, 30), activation: str = "tanh",
                 coordinates: str = "distances", length: float = 1.0, symmetrize: bool = False,
                 max_permutations: int = 5040, cutoff: float = 1.0):
        super().__init__()
        if coordinates not in ("distances", "inverse_distances", "exponential"):
            raise ValueError(f"unknown coordinates {coordinates!r}")
        self.species = [_z(z) for z in species]
        self.n_atoms = len(self.species)
        if self.n_atoms < 2:
            raise ValueError("a first-generation potential needs at least two atoms")
        self.cutoff = float(cutoff)
        self.coordinates = coordinates
        self.length = float(length)
        self.register_buffer("_species", torch.tensor(self.species, dtype=torch.long), persistent=False)
        pairs = torch.triu_indices(self.n_atoms, self.n_atoms, 1)
        self.register_buffer("_pairs", pairs, persistent=False)
        n_in = pairs.shape[1]
        perms = like_atom_permutations(self.species, max_permutations) if symmetrize else [list(range(self.n_atoms))]
        index = {(a, b): k for k, (a, b) in enumerate(pairs.t().tolist())}
        table = [[index[(min(p[a], p[b]), max(p[a], p[b]))] for a, b in pairs.t().tolist()] for p in perms]
        self.register_buffer("_perm_pairs", torch.tensor(table, dtype=torch.long), persistent=False)
        layers, d = [], n_in
        for h in hidden:
            layers += [nn.Linear(d, int(h)), make_activation(activation)]
            d = int(h)
        layers.append(nn.Linear(d, 1))
        self.net = nn.Sequential(*layers)
        self.register_buffer("input_mean", torch.zeros(n_in))
        self.register_buffer("input_std", torch.ones(n_in))
        self.register_buffer("energy_shift", torch.zeros(()))
        self.register_buffer("energy_scale", torch.ones(()))

    def inputs(self, data: AtomicGraph) -> Tensor:
        b = data.num_graphs
        if not bool((data.n_atoms == self.n_atoms).all()):
            raise ValueError(f"NNP1G is built for {self.n_atoms} atoms; got {data.n_atoms.tolist()}")
        if not bool((data.atomic_numbers.reshape(b, self.n_atoms) == self._species).all()):
            raise ValueError("the atoms are not the elements of the model in its order")
        pos = data.pos.reshape(b, self.n_atoms, 3).to(data.model_dtype)
        i, j = self._pairs
        r = torch.linalg.norm(pos[:, j] - pos[:, i], dim=-1)
        if self.coordinates == "inverse_distances":
            return 1.0 / r
        if self.coordinates == "exponential":
            return torch.exp(-r / self.length)
        return r

    def forward(self, data: AtomicGraph) -> dict:
        x = self.inputs(data)[:, self._perm_pairs]
        x = (x - self.input_mean.to(x.dtype)) / self.input_std.to(x.dtype)
        e = self.net(x).squeeze(-1).mean(-1)
        energy = self.energy_shift.to(e.dtype) + self.energy_scale.to(e.dtype) * e
        node = (energy / self.n_atoms)[data.batch]
        return {"node_energy": node, "energy": self.aggregate_energy(node, data)}

    @torch.no_grad()
    def fit_scaling(self, graphs: Iterable[AtomicGraph]) -> None:
        xs, es = [], []
        for data in graphs:
            xs.append(self.inputs(data)[:, self._perm_pairs].reshape(-1, self._pairs.shape[1]).double())
            if data.energy is not None:
                es.append(data.energy.double())
        x = torch.cat(xs)
        dt = self.input_mean.dtype
        self.input_mean.copy_(x.mean(0).to(dt))
        self.input_std.copy_(x.std(0).clamp(min=1e-12).to(dt))
        if es:
            e = torch.cat(es)
            self.energy_shift.copy_(e.mean().to(dt))
            self.energy_scale.copy_((e.std() if e.numel() > 1 else e.new_ones(())).clamp(min=1e-12).to(dt))

    @classmethod
    def from_config(cls, cfg) -> "NNP1G":
        e = dict(cfg.extra or {})
        return cls(e["species"], hidden=e.get("hidden", (30, 30)), activation=e.get("activation", "tanh"),
                   coordinates=e.get("coordinates", "distances"), length=float(e.get("length", 1.0)),
                   symmetrize=bool(e.get("symmetrize", False)), max_permutations=int(e.get("max_permutations", 5040)),
                   cutoff=float(cfg.cutoff))
