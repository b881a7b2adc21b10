"""OPLS (Jorgensen, Maxwell & Tirado-Rives, JACS 118, 11225 (1996)): harmonic bonds and angles,
Fourier proper dihedrals, ``V2`` impropers at trigonal centres, and Coulomb plus 12-6
Lennard-Jones between atoms three or more bonds apart (geometric mixing, 1-4 pairs scaled by the
library's fudge factors), on a fixed topology bound to the model.

The parameter library (``OPLSLibrary``), its sources (the shipped ``.frc`` variants ``oplsaa``,
``oplsaa-1996``, ``lopls``, ``CL&P``, ``oplsaa+``, any ``.frc`` path, or the native JSON), the
bonded-type resolution rules (exact before wildcard, SEAMM's improper precedence), the trainable
parameter groups, the total-charge projection and the per-term energy outputs follow the reference
(``src/xnn/ffnn/models/oplslib.py``, ``opls.py:149-1115``). Energies are eV (kcal/mol x
4.184 / 96.48533212331), lengths Å, angles radians; Coulomb constant 14.399645307997487 eV Å.
"""
from __future__ import annotations

import ast
import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence, Union

import torch
from torch import Tensor, nn
from torch.nn import Parameter, ParameterDict

from ..data import AtomicGraph
from ..data.elements import ATOMIC_NUMBERS
from ..models.base import InteratomicPotential
from ..models.fast import resolve_use_fast
from ..models.registry import register_model
from ..ops.scatter import scatter_sum
from .frc import WILDCARD as FRC_WILDCARD
from .frc import read_forcefield
from .geometry import (TINY, angle_theta, batch_index, dihedral_cos, geometric_mean, half_edges, pair_vectors,
                       quintic_switch)
from .topology import MolecularTopology, read_topology

KCAL_TO_EV = 4.336410424180094e-2
KE = 14.399645307997487
DEG = math.pi / 180.0
WILDCARD = "X"
_TERMS = ("nonbond", "bond", "angle", "torsion", "oop")
GROUPS = ("charge", "sigma", "epsilon", "bond_k", "bond_r0", "angle_k", "angle_theta0", "dihedral_v", "improper_v2")
MAX_Z = 100


def fourier_to_rb(v: Sequence[float]) -> list:
    """OPLS ``(V0..V4)`` to Ryckaert-Bellemans ``(C0..C5)`` (``psi = phi - 180``)."""
    v0, v1, v2, v3, v4 = (float(x) for x in v)
    return [v0 + v2 + 0.5 * (v1 + v3), 0.5 * (-v1 + 3.0 * v3), -v2 + 4.0 * v4, -2.0 * v3, -4.0 * v4, 0.0]


def rb_to_fourier(c: Sequence[float]) -> list:
    cs = [float(x) for x in c] + [0.0] * (6 - len(c))
    if abs(cs[5]) > 1e-10:
        raise ValueError(f"C5 = {cs[5]} is not representable by the OPLS Fourier form")
    v3, v4 = -0.5 * cs[3], -0.25 * cs[4]
    v2 = -cs[2] - cs[4]
    v1 = -1.5 * cs[3] - 2.0 * cs[1]
    return [cs[0] - v2 - 0.5 * (v1 + v3), v1, v2, v3, v4]


@dataclass
class OPLSLibrary:
    """Parameters in OPLS units (kcal/mol, Å, degrees), bonded tables keyed by class names joined
    with ``-`` (``X`` wildcard); ``E_bond = k (r - r0)^2``, ``E_angle = k (theta - theta0)^2``,
    dihedral ``v = [V0..V4]``, improper ``V2 / 2 (1 - cos 2 phi)`` with the centre third."""
    atom_types: dict = field(default_factory=dict)
    bond_types: dict = field(default_factory=dict)
    angle_types: dict = field(default_factory=dict)
    dihedral_types: dict = field(default_factory=dict)
    improper_types: dict = field(default_factory=dict)
    fudge_lj: float = 0.5
    fudge_qq: float = 0.5
    name: str = "opls"
    references: list = field(default_factory=list)
    templates: dict = field(default_factory=dict)
    fragments: dict = field(default_factory=dict)
    metadata: dict = field(default_factory=dict)
    notes: list = field(default_factory=list)

    def cls(self, type_name: str, term: str = "bond") -> str:
        e = self.atom_types[type_name]
        return str(e.get(f"cls_{term}", e.get("cls", type_name)))

    def save(self, path: Union[str, Path]) -> None:
        data = {k: getattr(self, k) for k in ("name", "references", "fudge_lj", "fudge_qq", "atom_types", "bond_types",
                                              "angle_types", "dihedral_types", "improper_types", "templates",
                                              "fragments", "metadata")}
        Path(path).write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")


def resolve_bond_type(table: dict, a: str, b: str) -> Optional[str]:
    return next((k for k in (f"{a}-{b}", f"{b}-{a}") if k in table), None)


def resolve_angle_type(table: dict, a: str, b: str, c: str) -> Optional[str]:
    return next((k for k in (f"{a}-{b}-{c}", f"{c}-{b}-{a}") if k in table), None)


def resolve_dihedral_type(table: dict, a: str, b: str, c: str, d: str) -> Optional[str]:
    """The matching key (either direction, ``X`` any class) with the most explicit positions,
    ties broken alphabetically."""
    quad, best, score = (a, b, c, d), None, -1
    for key in table:
        pat = tuple(key.split("-"))
        if len(pat) != 4:
            continue
        for cand in (quad, quad[::-1]):
            if all(p == WILDCARD or p == q for p, q in zip(pat, cand)):
                s = sum(p != WILDCARD for p in pat)
                if s > score or (s == score and key < best):
                    best, score = key, s
    return best


def improper_key(i: str, j: str, k: str, l: str) -> str:
    a, b, c = sorted((i, j, l))
    return f"{a}-{b}-{k}-{c}"


def resolve_improper_type(table: dict, i: str, j: str, k: str, l: str) -> Optional[str]:
    """Centre ``k``: exact outer triple, then one, two and three outer wildcards."""
    X = WILDCARD
    for p in ((i, j, l), (X, j, l), (i, X, l), (i, j, X), (X, X, l), (X, j, X), (i, X, X), (X, X, X)):
        key = improper_key(p[0], p[1], k, p[2])
        if key in table:
            return key
    return None


_UNSUPPORTED = ("simple_fourier_angle", "tabulated_angle", "quartic_bond", "quartic_angle", "torsion_1", "torsion_3",
                "buckingham", "nonbond(9-6)", "wilson_out_of_plane")


def from_forcefield(ff, strict: bool = True) -> OPLSLibrary:
    """An :class:`OPLSLibrary` from a resolved ``.frc`` variant of the OPLS functional form."""
    lib = OPLSLibrary(name=ff.name, metadata=dict(ff.metadata), templates=dict(ff.templates),
                      fragments=dict(ff.fragments), references=[r.text for r in ff.references_used()])
    extra = {k: len(ff.sections[k]) for k in ff.sections if k in _UNSUPPORTED}
    if extra:
        if strict:
            raise ValueError(f"force field {ff.name!r} uses functional forms the OPLS model does not implement: "
                             f"{extra} (section: rows). Pass strict=False to load it without those sections, "
                             "if your structures use none of the affected types")
        lib.notes += [f"ignored section {k} ({n} rows): functional form not implemented by the OPLS model"
                      for k, n in extra.items()]
    if "nonbond(12-6)" in ff.sections and ff.combination() != "geometric":
        raise ValueError(f"force field {ff.name!r} uses the {ff.combination()!r} combination rule; OPLS requires geometric")
    for name, at in ff.atom_types.items():
        e = {f"cls_{t}": ff.equivalent(name, t) for t in _TERMS}
        e["cls"] = e["cls_bond"]
        e["element"] = ATOMIC_NUMBERS.get(str(at.get("El", "")), 0)
        e["mass"] = float(at.get("Mass", 0.0))
        try:
            e["connections"] = int(at.get("connections", 0))
        except (TypeError, ValueError):
            e["connections"] = 0
        e["comment"] = str(at.get("Comment", ""))
        e["charge"] = ff.charge(name)
        lj = ff.nonbond(name)
        if lj is None:
            lj = (0.0, 0.0)
            lib.notes.append(f"atom type {name} has no nonbond(12-6) entry; sigma = epsilon = 0")
        e["sigma"], e["epsilon"] = float(lj[0]), float(lj[1])
        lib.atom_types[name] = e

    def key(k):
        return "-".join(WILDCARD if x == FRC_WILDCARD else x for x in k)
    for k, r in ff.rows("quadratic_bond").items():
        lib.bond_types[key(k)] = {"k": float(r.values["K2"]), "r0": float(r.values["R0"])}
    for k, r in ff.rows("quadratic_angle").items():
        lib.angle_types[key(k)] = {"k": float(r.values["K2"]), "theta0": float(r.values["Theta0"])}
    for k, r in ff.rows("torsion_opls").items():
        v = r.values
        lib.dihedral_types[key(k)] = {"v": [0.0, float(v["V1"]), float(v["V2"]), float(v["V3"]), float(v.get("V4", 0.0))]}
    for k, r in ff.rows("improper_opls").items():
        lib.improper_types[key(k)] = {"v2": float(r.values["V2"])}
    return lib


def read_opls(source: Union[str, Path], strict: bool = True) -> OPLSLibrary:
    """A library from native JSON, or a ``.frc`` spec (shipped variant name, path, ``path:variant``)."""
    s = str(source)
    if s.lower().endswith(".json"):
        d = json.loads(Path(s).read_text())
        return OPLSLibrary(atom_types=d.get("atom_types", {}), bond_types=d.get("bond_types", {}),
                           angle_types=d.get("angle_types", {}), dihedral_types=d.get("dihedral_types", {}),
                           improper_types=d.get("improper_types", {}), fudge_lj=float(d.get("fudge_lj", 0.5)),
                           fudge_qq=float(d.get("fudge_qq", 0.5)), name=d.get("name", Path(s).stem),
                           references=list(d.get("references", [])), templates=dict(d.get("templates", {})),
                           fragments=dict(d.get("fragments", {})), metadata=dict(d.get("metadata", {})))
    return from_forcefield(read_forcefield(s), strict=strict)


def builtin_library(name: str = "oplsaa", strict: bool = True) -> OPLSLibrary:
    return read_opls(name, strict=strict)


def split_trainable(trainable) -> tuple:
    """``(force-field groups, atom_ref trainable)``."""
    if isinstance(trainable, str):
        if trainable.lower() == "all":
            return "all", True
        return ((), True) if trainable == "atom_ref" else (trainable, False)
    return tuple(g for g in trainable if g != "atom_ref"), "atom_ref" in trainable


def _groups(trainable, known) -> set:
    s = (set(known) if trainable.lower() == "all" else {trainable}) if isinstance(trainable, str) else set(trainable)
    unknown = s - set(known)
    if unknown:
        raise ValueError(f"unknown trainable group(s) {sorted(unknown)}; available: {list(known)}")
    return s


class ChargeConstraints(nn.Module):
    """Linear total-charge constraints ``counts . charge = total`` (one row per bound molecule):
    ``charges`` is the ``charge`` parameter minus its minimum-norm correction onto them."""

    def __init__(self, n_types: int):
        super().__init__()
        dt = torch.get_default_dtype()
        self.register_buffer("charge_rows", torch.zeros(0, n_types, dtype=dt), persistent=False)
        self.register_buffer("charge_totals", torch.zeros(0, dtype=dt), persistent=False)
        self.register_buffer("charge_proj", torch.zeros(n_types, 0, dtype=dt), persistent=False)

    def constrain_charges(self, counts: Tensor, total: float) -> None:
        row = counts.detach().to(self.charge_rows).reshape(1, -1)
        self.charge_rows = torch.cat([self.charge_rows, row])
        self.charge_totals = torch.cat([self.charge_totals, row.new_tensor([float(total)])])
        self.charge_proj = torch.linalg.pinv(self.charge_rows)

    def project(self, q: Tensor) -> Tensor:
        if self.charge_rows.shape[0] == 0:
            return q
        return q - self.charge_proj @ (self.charge_rows @ q - self.charge_totals)


class OPLSForceField(ChargeConstraints):
    """The library as dense parameter tensors (eV, Å, rad) in a ``ParameterDict``: ``charge``,
    ``sigma``, ``epsilon`` per atom type; ``bond_k``, ``bond_r0``, ``angle_k``, ``angle_theta0``,
    ``dihedral_v (ND, 5)``, ``improper_v2`` per bonded type. Shareable by several models."""

    def __init__(self, library: Union[OPLSLibrary, str, Path], trainable=()):
        lib = library if isinstance(library, OPLSLibrary) else read_opls(str(library))
        super().__init__(len(lib.atom_types))
        dt = torch.get_default_dtype()
        train = _groups(trainable, GROUPS)
        self.name, self.fudge_lj, self.fudge_qq = lib.name, float(lib.fudge_lj), float(lib.fudge_qq)
        self.type_names = list(lib.atom_types)
        self._type_index = {n: i for i, n in enumerate(self.type_names)}
        self.type_cls = [lib.cls(n, "bond") for n in self.type_names]
        self.type_cls_angle = [lib.cls(n, "angle") for n in self.type_names]
        self.type_cls_torsion = [lib.cls(n, "torsion") for n in self.type_names]
        self.type_cls_oop = [lib.cls(n, "oop") for n in self.type_names]
        self.templates, self.fragments = dict(lib.templates), dict(lib.fragments)
        at = [lib.atom_types[n] for n in self.type_names]
        self.register_buffer("type_z", torch.tensor([int(a["element"]) for a in at], dtype=torch.long))
        self.register_buffer("type_mass", torch.tensor([float(a.get("mass", 0.0)) for a in at], dtype=dt))
        self._tables = {"bond": dict(lib.bond_types), "angle": dict(lib.angle_types),
                        "dihedral": dict(lib.dihedral_types), "improper": dict(lib.improper_types)}
        self.bond_keys, self.angle_keys = list(lib.bond_types), list(lib.angle_types)
        self.dihedral_keys, self.improper_keys = list(lib.dihedral_types), list(lib.improper_types)
        self._index = {t: {k: i for i, k in enumerate(keys)} for t, keys in
                       (("bond", self.bond_keys), ("angle", self.angle_keys), ("dihedral", self.dihedral_keys),
                        ("improper", self.improper_keys))}
        self.params = ParameterDict()

        def make(name, values, shape=None):
            t = torch.tensor(values, dtype=dt)
            self.params[name] = Parameter(t.reshape(shape) if shape else t, requires_grad=name in train)
        make("charge", [float(a["charge"]) for a in at])
        make("sigma", [float(a["sigma"]) for a in at])
        make("epsilon", [float(a["epsilon"]) * KCAL_TO_EV for a in at])
        make("bond_k", [float(lib.bond_types[k]["k"]) * KCAL_TO_EV for k in self.bond_keys])
        make("bond_r0", [float(lib.bond_types[k]["r0"]) for k in self.bond_keys])
        make("angle_k", [float(lib.angle_types[k]["k"]) * KCAL_TO_EV for k in self.angle_keys])
        make("angle_theta0", [float(lib.angle_types[k]["theta0"]) * DEG for k in self.angle_keys])
        make("dihedral_v", [[float(x) * KCAL_TO_EV for x in (list(lib.dihedral_types[k]["v"]) + [0.0] * 5)[:5]]
                            for k in self.dihedral_keys], (len(self.dihedral_keys), 5))
        make("improper_v2", [float(lib.improper_types[k]["v2"]) * KCAL_TO_EV for k in self.improper_keys])

    @property
    def charges(self) -> Tensor:
        return self.project(self.params["charge"])

    def type_index(self, name: str) -> int:
        if name not in self._type_index:
            raise KeyError(f"atom type {name!r} is not in library {self.name!r}")
        return self._type_index[name]

    def resolve_bond(self, a, b) -> int:
        k = resolve_bond_type(self._tables["bond"], a, b)
        if k is None:
            raise KeyError(f"no bond type {a}-{b} in library {self.name!r}")
        return self._index["bond"][k]

    def resolve_angle(self, a, b, c) -> int:
        k = resolve_angle_type(self._tables["angle"], a, b, c)
        if k is None:
            raise KeyError(f"no angle type {a}-{b}-{c} in library {self.name!r}")
        return self._index["angle"][k]

    def resolve_dihedral(self, a, b, c, d) -> int:
        k = resolve_dihedral_type(self._tables["dihedral"], a, b, c, d)
        if k is None:
            raise KeyError(f"no dihedral type {a}-{b}-{c}-{d} in library {self.name!r}")
        return self._index["dihedral"][k]

    def resolve_improper(self, *args) -> int:
        if len(args) == 1:
            if args[0] not in self._index["improper"]:
                raise KeyError(f"no improper type {args[0]!r} in library {self.name!r}")
            return self._index["improper"][args[0]]
        k = resolve_improper_type(self._tables["improper"], *args)
        if k is None:
            i, j, c, l = args
            raise KeyError(f"no improper type for {i}-{j}-{c}-{l} (center {c}) in library {self.name!r}")
        return self._index["improper"][k]

    def improper_defined(self, i, j, k, l) -> bool:
        return resolve_improper_type(self._tables["improper"], i, j, k, l) is not None

    def export_library(self) -> OPLSLibrary:
        """The current parameters as a library in OPLS units."""
        P = {k: v.detach().cpu() for k, v in self.params.items()}
        P["charge"] = self.charges.detach().cpu()
        lib = OPLSLibrary(name=self.name, fudge_lj=self.fudge_lj, fudge_qq=self.fudge_qq,
                          templates=dict(self.templates), fragments=dict(self.fragments))
        for i, n in enumerate(self.type_names):
            lib.atom_types[n] = {"cls": self.type_cls[i], "cls_nonbond": n, "cls_bond": self.type_cls[i],
                                 "cls_angle": self.type_cls_angle[i], "cls_torsion": self.type_cls_torsion[i],
                                 "cls_oop": self.type_cls_oop[i], "element": int(self.type_z[i]),
                                 "mass": float(self.type_mass[i]), "charge": float(P["charge"][i]),
                                 "sigma": float(P["sigma"][i]), "epsilon": float(P["epsilon"][i]) / KCAL_TO_EV}
        for i, k in enumerate(self.bond_keys):
            lib.bond_types[k] = {"k": float(P["bond_k"][i]) / KCAL_TO_EV, "r0": float(P["bond_r0"][i])}
        for i, k in enumerate(self.angle_keys):
            lib.angle_types[k] = {"k": float(P["angle_k"][i]) / KCAL_TO_EV, "theta0": float(P["angle_theta0"][i]) / DEG}
        for i, k in enumerate(self.dihedral_keys):
            lib.dihedral_types[k] = {"v": [float(x) / KCAL_TO_EV for x in P["dihedral_v"][i]]}
        for i, k in enumerate(self.improper_keys):
            lib.improper_types[k] = {"v2": float(P["improper_v2"][i]) / KCAL_TO_EV}
        return lib


class FixedTopologyPotential(InteratomicPotential):
    """Shared machinery of the fixed-topology force fields: integer index buffers of the bound
    topology, batch checks (conformers of that system), per-element reference energies and the
    once-per-pair nonbonded sum with exclusions and the quintic switch."""

    #: whether one evaluation can be recorded as a CUDA graph (no host reads, fixed shapes)
    graph_capturable = True

    def _check_batch(self, data: AtomicGraph) -> tuple:
        n = int(self.top_type.shape[0])
        if data.pos.is_cuda and torch.cuda.is_current_stream_capturing():
            return data.num_nodes, data.num_graphs, n          # checked when the graph was recorded
        if not bool((data.n_atoms == n).all()):
            raise ValueError(f"every structure must have the bound topology's {n} atoms (got {data.n_atoms.tolist()})")
        if not bool((data.atomic_numbers == self.top_z.repeat(data.num_graphs)).all()):
            raise ValueError("atomic numbers do not match the bound topology's element sequence")
        return data.num_nodes, data.num_graphs, n

    def _buf(self, name: str, rows, width: int) -> None:
        t = torch.tensor(rows, dtype=torch.long).reshape(-1, width) if width > 1 else torch.tensor(rows, dtype=torch.long)
        self.register_buffer(name, t.t().contiguous() if width > 1 else t)

    def _pairs_once(self, data, excl_index: Tensor, n: int):
        return half_edges(data, excl_index, n, self.__dict__.setdefault("_exclusion_keys", {}))

    @property
    def masses(self) -> Tensor:
        return self.ff.type_mass[self.top_type]

    def set_use_fast(self, use_fast) -> "FixedTopologyPotential":
        """Accepted for the common model interface; the bonded and nonbonded terms here have one
        formulation (index-gather PyTorch ops, capturable in a CUDA graph), so the mode changes
        nothing numerically."""
        self.use_fast = resolve_use_fast(use_fast)
        return self


@register_model("opls")
class OPLS(FixedTopologyPotential):
    """An OPLS library bound to one molecular topology; ``forward`` takes any batch of its
    conformers. Outputs ``node_energy``, ``energy``, ``charges``, ``node_features`` and the
    per-structure terms ``e_bond``, ``e_angle``, ``e_torsion``, ``e_improper``, ``e_lj``,
    ``e_coulomb``, ``e_lj14``, ``e_coulomb14``, ``e_ref``."""

    def __init__(self, ffield, topology, *, cutoff: float = 10.0, switch_width: float = 0.0,
                 fudge_lj: Optional[float] = None, fudge_qq: Optional[float] = None, trainable=(),
                 keep_intermediates: bool = False, auto_impropers: bool = True, constrain_charge=True,
                 use_fast="auto", atomic_energies=None):
        super().__init__()
        groups, ref_train = split_trainable(trainable)
        self.ff = ffield if isinstance(ffield, OPLSForceField) else OPLSForceField(ffield, trainable=groups)
        self.atom_ref = nn.Embedding(MAX_Z, 1)
        nn.init.zeros_(self.atom_ref.weight)
        self.atom_ref.weight.requires_grad_(ref_train)
        self.auto_impropers = bool(auto_impropers)
        self.cutoff, self.switch_width = float(cutoff), float(switch_width)
        if not 0.0 <= self.switch_width < self.cutoff:
            raise ValueError("switch_width must satisfy 0 <= switch_width < cutoff")
        self.fudge_lj = self.ff.fudge_lj if fudge_lj is None else float(fudge_lj)
        self.fudge_qq = self.ff.fudge_qq if fudge_qq is None else float(fudge_qq)
        self.keep_intermediates = bool(keep_intermediates)
        self.intermediates: dict = {}
        self.node_feature_dim = 1
        self.use_fast = resolve_use_fast(use_fast)
        self._bind(topology if isinstance(topology, MolecularTopology) else read_topology(topology))
        self.species = sorted({int(z) for z in self.top_z.tolist()})
        if atomic_energies is not None:
            set_atomic_energies(self, atomic_energies)
        if constrain_charge is not False:
            q = self.ff.params["charge"].detach()
            counts = torch.bincount(self.top_type, minlength=q.shape[0]).to(q)
            self.ff.constrain_charges(counts, float(counts @ q) if constrain_charge is True else float(constrain_charge))

    def _bind(self, top: MolecularTopology) -> None:
        self.topology, ff, missing = top, self.ff, []

        def get(fn, *a):
            try:
                return fn(*a)
            except KeyError as err:
                if str(err.args[0]) not in missing:
                    missing.append(str(err.args[0]))
                return 0
        t = [get(ff.type_index, nm) for nm in top.types]
        cb, ca = [ff.type_cls[i] for i in t], [ff.type_cls_angle[i] for i in t]
        ct, co = [ff.type_cls_torsion[i] for i in t], [ff.type_cls_oop[i] for i in t]
        bt = [get(ff.resolve_bond, cb[i], cb[j]) for i, j in top.bonds]
        at = [get(ff.resolve_angle, ca[i], ca[j], ca[k]) for i, j, k in top.angles]
        dt = [get(ff.resolve_dihedral, ct[i], ct[j], ct[k], ct[l]) for i, j, k, l in top.dihedrals]
        imps = [tuple(int(x) for x in im) for im in top.impropers]
        if top.improper_keys:
            it = [get(ff.resolve_improper, k) for k in top.improper_keys]
        elif imps:
            it = [get(ff.resolve_improper, co[i], co[j], co[k], co[l]) for i, j, k, l in imps]
        elif self.auto_impropers:
            # one improper per three-connected centre, outer atoms ascending, centre third
            nbr: dict = {}
            for i, j in top.bonds:
                nbr.setdefault(i, []).append(j)
                nbr.setdefault(j, []).append(i)
            it = []
            for m, nb in sorted(nbr.items()):
                if len(nb) == 3:
                    a, b, c = sorted(nb)
                    if ff.improper_defined(co[a], co[b], co[m], co[c]):
                        imps.append((a, b, m, c))
                        it.append(ff.resolve_improper(co[a], co[b], co[m], co[c]))
        else:
            it = []
        if missing:
            raise KeyError("the topology needs parameters the library does not provide:\n  " + "\n  ".join(missing))
        self._buf("top_type", t, 1)
        self.register_buffer("top_z", ff.type_z[self.top_type].clone())
        self._buf("bond_index", top.bonds, 2)
        self._buf("bond_type", bt, 1)
        self._buf("angle_index", top.angles, 3)
        self._buf("angle_type", at, 1)
        self._buf("dihedral_index", top.dihedrals, 4)
        self._buf("dihedral_type", dt, 1)
        self.impropers = imps
        self._buf("improper_index", imps, 4)
        self._buf("improper_type", it, 1)
        self._buf("pair14_index", top.pairs14, 2)
        self._buf("excl_index", sorted(set(top.exclusions) | set(top.pairs14)), 2)

    @staticmethod
    def _lj_coulomb(sig_i, sig_j, eps_i, eps_j, q_i, q_j, r, r2):
        sig, eps = geometric_mean(sig_i, sig_j), geometric_mean(eps_i, eps_j)
        s6 = (sig * sig / (r2 + TINY)) ** 3
        return 4.0 * eps * (s6 * s6 - s6), KE * q_i * q_j / r

    def forward(self, data: AtomicGraph) -> dict:
        N, B, n = self._check_batch(data)
        P = self.ff.params
        t = self.top_type.repeat(B)
        q = self.ff.charges[t]
        bi, ai = batch_index(self.bond_index, n, B), batch_index(self.angle_index, n, B)
        di, ii = batch_index(self.dihedral_index, n, B), batch_index(self.improper_index, n, B)
        pi = batch_index(self.pair14_index, n, B)
        # bonds, angles
        btype = self.bond_type.repeat(B)
        bv = pair_vectors(data, bi[0], bi[1])
        br = torch.sqrt((bv * bv).sum(1) + TINY)
        e_bond = P["bond_k"][btype] * (br - P["bond_r0"][btype]) ** 2
        e_bond_node = scatter_sum(0.5 * e_bond, bi[0], N) + scatter_sum(0.5 * e_bond, bi[1], N)
        atype = self.angle_type.repeat(B)
        theta = angle_theta(data, ai)
        e_angle = P["angle_k"][atype] * (theta - P["angle_theta0"][atype]) ** 2
        e_angle_node = scatter_sum(e_angle, ai[1], N)
        # proper dihedrals: V0 + 1/2 [V1 (1 + c) + V2 (1 - c2) + V3 (1 + c3) + V4 (1 - c4)]
        c1 = dihedral_cos(data, di)
        c2 = 2.0 * c1 * c1 - 1.0
        c3, c4 = c1 * (4.0 * c1 * c1 - 3.0), 2.0 * c2 * c2 - 1.0
        vd = P["dihedral_v"][self.dihedral_type.repeat(B)]
        e_tors = vd[:, 0] + 0.5 * (vd[:, 1] * (1.0 + c1) + vd[:, 2] * (1.0 - c2) + vd[:, 3] * (1.0 + c3)
                                   + vd[:, 4] * (1.0 - c4))
        e_tors_node = scatter_sum(e_tors, di[1], N)
        ci = dihedral_cos(data, ii)
        e_impr = 0.5 * P["improper_v2"][self.improper_type.repeat(B)] * (1.0 - (2.0 * ci * ci - 1.0))
        e_impr_node = scatter_sum(e_impr, ii[2], N)
        # scaled 1-4 pairs, exact
        pv = pair_vectors(data, pi[0], pi[1])
        pr2 = (pv * pv).sum(1)
        pr = torch.sqrt(pr2 + TINY)
        ta, tb = t[pi[0]], t[pi[1]]
        lj14, c14 = self._lj_coulomb(P["sigma"][ta], P["sigma"][tb], P["epsilon"][ta], P["epsilon"][tb],
                                     q[pi[0]], q[pi[1]], pr, pr2)
        lj14, c14 = self.fudge_lj * lj14, self.fudge_qq * c14
        e_lj14_node = scatter_sum(0.5 * lj14, pi[0], N) + scatter_sum(0.5 * lj14, pi[1], N)
        e_c14_node = scatter_sum(0.5 * c14, pi[0], N) + scatter_sum(0.5 * c14, pi[1], N)
        # nonbonded over the neighbour list minus exclusions
        src, dst, _vec, r2, half, keep = self._pairs_once(data, self.excl_index, n)
        r = torch.sqrt(r2 + TINY)
        sig, eps = P["sigma"][t], P["epsilon"][t]
        lj, coul = self._lj_coulomb(sig[src], sig[dst], eps[src], eps[dst], q[src], q[dst], r, r2)
        w = keep.to(r.dtype) * half * quintic_switch(r, self.cutoff, self.switch_width)
        h_lj, h_c = 0.5 * w * lj, 0.5 * w * coul
        e_lj_node = scatter_sum(h_lj, src, N) + scatter_sum(h_lj, dst, N)
        e_c_node = scatter_sum(h_c, src, N) + scatter_sum(h_c, dst, N)
        e_ref_node = self.atom_ref(data.atomic_numbers).squeeze(-1)
        node = (e_bond_node + e_angle_node + e_tors_node + e_impr_node + e_lj_node + e_c_node + e_lj14_node
                + e_c14_node + e_ref_node)
        if self.keep_intermediates:
            self.intermediates = dict(bond_r=br, e_bond=e_bond, angle_theta=theta, e_angle=e_angle, dihedral_cos=c1,
                                      e_torsion=e_tors, improper_cos=ci, e_improper=e_impr, pair14_r=pr, e_lj14=lj14,
                                      e_coulomb14=c14, type_index=t, nb_r=r, nb_weight=w, nb_lj=lj, nb_coulomb=coul)
        agg = lambda x: self.aggregate_energy(x, data)  # noqa: E731
        return {"node_energy": node, "energy": agg(node), "charges": q, "node_features": q.unsqueeze(1),
                "e_bond": agg(e_bond_node), "e_angle": agg(e_angle_node), "e_torsion": agg(e_tors_node),
                "e_improper": agg(e_impr_node), "e_lj": agg(e_lj_node), "e_coulomb": agg(e_c_node),
                "e_lj14": agg(e_lj14_node), "e_coulomb14": agg(e_c14_node), "e_ref": agg(e_ref_node)}

    def export_library(self) -> OPLSLibrary:
        return self.ff.export_library()

    @classmethod
    def from_config(cls, cfg) -> "OPLS":
        e = dict(cfg.extra or {})
        library = e.get("library")
        if library is None:
            raise ValueError("OPLS needs a parameter library: set model.library to 'oplsaa', 'lopls', 'CL&P', "
                             "a .frc path or a native JSON path")
        return cls(library, topology_from_options(e, "OPLS"), cutoff=float(cfg.cutoff),
                   switch_width=float(e.get("switch_width") or 0.0), fudge_lj=_floaty(e, "fudge_lj"),
                   fudge_qq=_floaty(e, "fudge_qq"), trainable=_listy(e.get("trainable")) or (),
                   constrain_charge=_constrain(e.get("constrain_charge", True)),
                   atomic_energies=e.get("atomic_energies"))


def _listy(v):
    if isinstance(v, str) and v.lstrip().startswith(("[", "(")):
        return ast.literal_eval(v)
    return v


def _floaty(e: dict, key: str):
    return None if e.get(key) is None else float(e[key])


def _constrain(v):
    if isinstance(v, str):
        v = {"true": True, "false": False}.get(v.strip().lower(), v)
        if isinstance(v, str):
            v = float(v)
    return v


def topology_from_options(e: dict, who: str) -> MolecularTopology:
    """A topology from ``topology`` (JSON path) or inline ``types`` + ``bonds`` (+ impropers)."""
    if e.get("topology") is not None:
        return read_topology(e["topology"])
    types, bonds = _listy(e.get("types")), _listy(e.get("bonds"))
    if types is None or bonds is None:
        raise ValueError(f"{who} needs a topology: set model.topology to a topology JSON path, or give "
                         "model.types and model.bonds inline")
    return MolecularTopology.from_bonds(types, bonds, impropers=_listy(e.get("impropers")) or (),
                                        improper_keys=_listy(e.get("improper_keys")) or (),
                                        bond_orders=_listy(e.get("bond_orders")), charges=_listy(e.get("charges")))


def set_atomic_energies(model, values) -> None:
    """``{Z or symbol: E0}`` into ``model.atom_ref``."""
    with torch.no_grad():
        for k, v in dict(values).items():
            z = int(k) if str(k).lstrip("-").isdigit() else ATOMIC_NUMBERS[str(k)]
            model.atom_ref.weight[z, 0] = float(v)
