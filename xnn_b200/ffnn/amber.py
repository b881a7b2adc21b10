"""AMBER (Cornell et al., JACS 117, 5179 (1995)): harmonic bonds and angles, phased Fourier
torsions ``sum K [1 + cos(n phi - gamma)]``, impropers of the same form centred on the third atom,
``eps_ij [(R*_ij / r)^12 - 2 (R*_ij / r)^6]`` van der Waals with ``R*_ij = R*_i + R*_j`` and
``eps_ij = sqrt(eps_i eps_j)``, Coulomb with the AMBER constant ``18.2223^2`` kcal Å / (mol e^2), 1-4
pairs scaled by 1/2 and 1/1.2. Charges belong to the structure (residue templates), not to the
atom types: per-atom, optionally trainable with the total held.

Library fields, ``ff94`` (``amber.frc``), improper placement by the AMBER builder's rules
(``match_improper``: explicit patterns preferred, the last explicit or the first wildcard match,
template order between equal positions) and the outputs follow the reference
(``src/xnn/ffnn/models/amberlib.py``, ``amber.py``).
"""
from __future__ import annotations

import itertools
import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence, Union

import torch
from torch import Tensor, nn
from torch.nn import Parameter, ParameterDict

from ..data import AtomicGraph
from ..data.elements import ATOMIC_NUMBERS, SYMBOLS
from ..models.fast import resolve_use_fast
from ..models.registry import register_model
from ..ops.scatter import scatter_sum
from .frc import read_forcefield
from .geometry import TINY, angle_theta, batch_index, dihedral_cos_sin, geometric_mean, pair_vectors, quintic_switch
from .opls import (DEG, KCAL_TO_EV, MAX_Z, WILDCARD, FixedTopologyPotential, _constrain, _floaty, _groups, _listy,
                   resolve_angle_type, resolve_bond_type, resolve_dihedral_type, set_atomic_energies,
                   topology_from_options)
from .topology import MolecularTopology, read_topology

SCALE_14_VDW, SCALE_14_COULOMB = 0.5, 1.0 / 1.2
TWO_SIXTH = 2.0 ** (1.0 / 6.0)
KE_KCAL = 18.2223 ** 2
KE = KE_KCAL * KCAL_TO_EV
MAX_TERMS, MAX_IMPROPER_TERMS = 4, 2
GROUPS = ("rstar", "epsilon", "bond_k", "bond_r0", "angle_k", "angle_theta0", "dihedral_k", "improper_k")
MODEL_GROUPS = ("charge", "atom_ref")
_TERMS = ("nonbond", "bond", "angle", "torsion", "oop")


@dataclass
class AmberLibrary:
    """kcal/mol, Å, degrees; ``rstar`` is half the like-pair minimum distance; torsion and
    improper rows ``{"terms": [[K, n, gamma], ...]}`` (improper ``I-J-K-L``, ``K`` central, ``L`` the
    distinguished outer atom)."""
    atom_types: dict = field(default_factory=dict)
    bond_types: dict = field(default_factory=dict)
    angle_types: dict = field(default_factory=dict)
    dihedral_types: dict = field(default_factory=dict)
    improper_types: dict = field(default_factory=dict)
    fudge_lj: float = SCALE_14_VDW
    fudge_qq: float = SCALE_14_COULOMB
    name: str = "amber"
    references: list = field(default_factory=list)
    templates: dict = field(default_factory=dict)
    fragments: dict = field(default_factory=dict)
    metadata: dict = field(default_factory=dict)
    notes: list = field(default_factory=list)

    def cls(self, type_name: str, term: str = "bond") -> str:
        return str(self.atom_types[type_name].get(f"cls_{term}", type_name))

    def residue_charges(self, name: str) -> dict:
        frag = self.fragments[name]
        return {str(a): float(q) for a, q in zip(frag.get("atom names", []), frag.get("charges", []))}

    def save(self, path: Union[str, Path]) -> None:
        data = {k: getattr(self, k) for k in ("name", "references", "fudge_lj", "fudge_qq", "atom_types", "bond_types",
                                              "angle_types", "dihedral_types", "improper_types", "templates",
                                              "fragments", "metadata")}
        Path(path).write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")


def _fits(pattern, types) -> bool:
    return all(p == WILDCARD or p == t for p, t in zip(pattern, types))


def match_improper(table: dict, center: str, outer: Sequence[tuple]):
    """``(key, (i, j, l))`` of the improper pattern for a centre and its three neighbours
    ``(index, type, element, order key)``, or ``None``. Explicit patterns beat wildcard ones (the
    last explicit match wins, else the first wildcard match in table order); equal positions are
    ordered by the residue-template order (explicit: equal types; wildcard: equal elements with
    ``L``, and always the two leading positions)."""
    best = None
    for key in table:
        pat = key.split("-")
        if len(pat) != 4 or pat[2] != center:
            continue
        wild = WILDCARD in (pat[0], pat[1], pat[3])
        if best is not None and wild:
            continue
        for a, b, c in itertools.permutations(outer):
            if not _fits((pat[0], pat[1], pat[3]), (a[1], b[1], c[1])):
                continue
            same = 1 if not wild else 2          # compare types (explicit) or elements (wildcard)
            if a[same] == c[same] and a[3] > c[3]:
                a, c = c, a
            if b[same] == c[same] and b[3] > c[3]:
                b, c = c, b
            if (a[1] == b[1] or wild) and a[3] > b[3]:
                a, b = b, a
            best = (key, (a[0], b[0], c[0]))
            break
    return best


def place_impropers(top: MolecularTopology, cls_oop: Sequence[str], elements: Sequence[str], table: dict):
    """One improper ``(i, j, centre, l)`` per three-connected atom with a matching pattern."""
    nbr: dict = {}
    for i, j in top.bonds:
        nbr.setdefault(i, []).append(j)
        nbr.setdefault(j, []).append(i)
    res = list(top.residues)

    def order(a):
        r = res[a] if a < len(res) else None
        return (-1, a) if r is None else (int(r[0]), int(r[1]))
    imps, keys = [], []
    for c in sorted(nbr):
        nb = sorted(nbr[c])
        if len(nb) != 3:
            continue
        found = match_improper(table, cls_oop[c], [(a, cls_oop[a], elements[a], order(a)) for a in nb])
        if found is not None:
            key, (i, j, l) = found
            imps.append((i, j, c, l))
            keys.append(key)
    return imps, keys


def resolve_improper_type(table: dict, i: str, j: str, k: str, l: str) -> Optional[str]:
    """Centre ``k``, distinguished ``l``: exact (either order of ``i, j``), then the first wildcard
    pattern in table order."""
    for key in (f"{i}-{j}-{k}-{l}", f"{j}-{i}-{k}-{l}"):
        if key in table:
            return key
    for cand in table:
        p = cand.split("-")
        if len(p) == 4 and p[2] == k and (_fits((p[0], p[1], p[3]), (i, j, l)) or _fits((p[0], p[1], p[3]), (j, i, l))):
            return cand
    return None


def _terms(values: dict, width: int) -> list:
    out = []
    for m in range(1, width + 1):
        k = values.get(f"K{m}")
        if k is None or k == "":
            break
        out.append([float(k), int(round(float(values.get(f"n{m}", 0)))), float(values.get(f"Phi0_{m}", 0.0))])
    return out


_UNSUPPORTED = ("simple_fourier_angle", "tabulated_angle", "quartic_bond", "quartic_angle", "torsion_1", "torsion_3",
                "torsion_opls", "improper_opls", "buckingham", "nonbond(9-6)", "wilson_out_of_plane")


def from_forcefield(ff, strict: bool = True) -> AmberLibrary:
    lib = AmberLibrary(name=ff.name, metadata=dict(ff.metadata), templates=dict(ff.templates),
                       fragments=dict(ff.fragments), references=[r.text for r in ff.references_used()])
    lib.fudge_lj = float(lib.metadata.get("scale_14_vdw", SCALE_14_VDW))
    lib.fudge_qq = float(lib.metadata.get("scale_14_coulomb", SCALE_14_COULOMB))
    extra = {k: len(ff.sections[k]) for k in ff.sections if k in _UNSUPPORTED}
    if extra:
        if strict:
            raise ValueError(f"force field {ff.name!r} uses functional forms the AMBER model does not implement: "
                             f"{extra}. Pass strict=False to load it without those sections")
        lib.notes += [f"ignored section {k} ({n} rows): functional form not implemented by the AMBER model"
                      for k, n in extra.items()]
    if "nonbond(12-6)" in ff.sections and ff.combination() != "arithmetic":
        raise ValueError(f"force field {ff.name!r} uses the {ff.combination()!r} combination rule; AMBER requires "
                         "arithmetic (Lorentz-Berthelot)")
    for name, at in ff.atom_types.items():
        e = {f"cls_{t}": ff.equivalent(name, t) for t in _TERMS}
        e["element"] = ATOMIC_NUMBERS.get(str(at.get("El", "")), 0)
        e["mass"] = float(at.get("Mass", 0.0))
        try:
            e["connections"] = int(at.get("connections", 0))
        except (TypeError, ValueError):
            e["connections"] = 0
        e["comment"] = str(at.get("Comment", ""))
        lj = ff.nonbond(name)
        if lj is None:
            lj = (0.0, 0.0)
            lib.notes.append(f"atom type {name} has no nonbond(12-6) entry; R* = epsilon = 0")
        e["rstar"], e["epsilon"] = float(lj[0]) * TWO_SIXTH / 2.0, float(lj[1])
        lib.atom_types[name] = e

    def key(k):
        return "-".join(WILDCARD if x == "*" else x for x in k)
    for k, r in ff.rows("quadratic_bond").items():
        lib.bond_types[key(k)] = {"k": float(r.values["K2"]), "r0": float(r.values["R0"])}
    for k, r in ff.rows("quadratic_angle").items():
        lib.angle_types[key(k)] = {"k": float(r.values["K2"]), "theta0": float(r.values["Theta0"])}
    for k, r in ff.rows("torsion_fourier").items():
        lib.dihedral_types[key(k)] = {"terms": _terms(r.values, MAX_TERMS)}
    for k, r in ff.rows("improper_fourier").items():
        lib.improper_types[key(k)] = {"terms": _terms(r.values, MAX_IMPROPER_TERMS)}
    return lib


def read_amber(source: Union[str, Path], strict: bool = True) -> AmberLibrary:
    s = str(source)
    if s.lower().endswith(".json"):
        d = json.loads(Path(s).read_text())
        return AmberLibrary(**{k: d.get(k, getattr(AmberLibrary, k, None)) for k in (
            "atom_types", "bond_types", "angle_types", "dihedral_types", "improper_types")},
            fudge_lj=float(d.get("fudge_lj", SCALE_14_VDW)), fudge_qq=float(d.get("fudge_qq", SCALE_14_COULOMB)),
            name=d.get("name", Path(s).stem), references=list(d.get("references", [])),
            templates=dict(d.get("templates", {})), fragments=dict(d.get("fragments", {})),
            metadata=dict(d.get("metadata", {})))
    return from_forcefield(read_forcefield(s), strict=strict)


def exact_trig(values: Tensor):
    """``cos``/``sin`` of phases with the values at multiples of 90 degrees snapped exact."""
    c, s = torch.cos(values), torch.sin(values)
    for t in (c, s):
        for target in (-1.0, 0.0, 1.0):
            t[(t - target).abs() < 1e-12] = target
    return c, s


def multiple_angles(c1: Tensor, s1: Tensor, n_max: int):
    """``(M, n_max)`` ``cos(n phi)``, ``sin(n phi)`` by the addition recurrences."""
    cs, ss = [c1], [s1]
    for _ in range(1, n_max):
        cs.append(cs[-1] * c1 - ss[-1] * s1)
        ss.append(ss[-1] * c1 + cs[-2] * s1)
    return torch.stack(cs, 1), torch.stack(ss, 1)


def register_periodic(module: nn.Module, prefix: str, rows: list, width: int, train: bool) -> None:
    """Fourier term slots ``(rows, width)`` of torsion-like rows on ``module``: the trainable
    ``params[prefix_k]`` and the fixed buffers ``prefix_n``, ``prefix_cos``, ``prefix_sin`` (of the
    phases) and ``prefix_mask`` (used slots)."""
    dt = torch.get_default_dtype()
    ks, ns, phs, ms = [], [], [], []
    for terms in rows:
        terms = list(terms)[:width]
        pad = width - len(terms)
        ks.append([float(t[0]) * KCAL_TO_EV for t in terms] + [0.0] * pad)
        ns.append([max(int(t[1]), 1) for t in terms] + [1] * pad)
        phs.append([float(t[2]) * DEG for t in terms] + [0.0] * pad)
        ms.append([1.0] * len(terms) + [0.0] * pad)
    module.params[f"{prefix}_k"] = Parameter(torch.tensor(ks, dtype=dt).reshape(len(rows), width), requires_grad=train)
    n = torch.tensor(ns, dtype=torch.long).reshape(len(rows), width)
    module.register_buffer(f"{prefix}_n", n)
    module.register_buffer(f"{prefix}_mask", torch.tensor(ms, dtype=dt).reshape(len(rows), width))
    c, s = exact_trig(torch.tensor(phs, dtype=torch.float64).reshape(len(rows), width))
    module.register_buffer(f"{prefix}_cos", c.to(dt))
    module.register_buffer(f"{prefix}_sin", s.to(dt))
    setattr(module, f"{prefix}_nmax", max(int(n.max()), 1) if n.numel() else 1)


def periodic_energy(module: nn.Module, prefix: str, c1: Tensor, s1: Tensor, types: Tensor) -> Tensor:
    """``sum_m K_m [1 + cos(n_m phi - gamma_m)]`` per row from ``cos phi``, ``sin phi``."""
    cn, sn = multiple_angles(c1, s1, getattr(module, f"{prefix}_nmax"))
    n = getattr(module, f"{prefix}_n")[types] - 1
    k = module.params[f"{prefix}_k"][types] * getattr(module, f"{prefix}_mask")[types]
    return (k * (1.0 + getattr(module, f"{prefix}_cos")[types] * torch.gather(cn, 1, n)
                 + getattr(module, f"{prefix}_sin")[types] * torch.gather(sn, 1, n))).sum(1)


class AmberForceField(nn.Module):
    def __init__(self, library: Union[AmberLibrary, str, Path], trainable=()):
        super().__init__()
        lib = library if isinstance(library, AmberLibrary) else read_amber(str(library))
        dt = torch.get_default_dtype()
        train = _groups(trainable, GROUPS)
        self.name, self.fudge_lj, self.fudge_qq = lib.name, float(lib.fudge_lj), float(lib.fudge_qq)
        self.type_names = list(lib.atom_types)
        self._type_index = {n: i for i, n in enumerate(self.type_names)}
        self.type_cls = [lib.cls(n, "bond") for n in self.type_names]
        self.type_cls_angle = [lib.cls(n, "angle") for n in self.type_names]
        self.type_cls_torsion = [lib.cls(n, "torsion") for n in self.type_names]
        self.type_cls_oop = [lib.cls(n, "oop") for n in self.type_names]
        self.templates, self.fragments, self.metadata = dict(lib.templates), dict(lib.fragments), dict(lib.metadata)
        at = [lib.atom_types[n] for n in self.type_names]
        self.register_buffer("type_z", torch.tensor([int(a["element"]) for a in at], dtype=torch.long))
        self.register_buffer("type_mass", torch.tensor([float(a.get("mass", 0.0)) for a in at], dtype=dt))
        self._tables = {"bond": dict(lib.bond_types), "angle": dict(lib.angle_types),
                        "dihedral": dict(lib.dihedral_types), "improper": dict(lib.improper_types)}
        self.bond_keys, self.angle_keys = list(lib.bond_types), list(lib.angle_types)
        self.dihedral_keys, self.improper_keys = list(lib.dihedral_types), list(lib.improper_types)
        self._index = {t: {k: i for i, k in enumerate(getattr(self, f"{t}_keys"))}
                       for t in ("bond", "angle", "dihedral", "improper")}
        self.params = ParameterDict()
        for name, vals in (("rstar", [float(a["rstar"]) for a in at]),
                           ("epsilon", [float(a["epsilon"]) * KCAL_TO_EV for a in at]),
                           ("bond_k", [float(lib.bond_types[k]["k"]) * KCAL_TO_EV for k in self.bond_keys]),
                           ("bond_r0", [float(lib.bond_types[k]["r0"]) for k in self.bond_keys]),
                           ("angle_k", [float(lib.angle_types[k]["k"]) * KCAL_TO_EV for k in self.angle_keys]),
                           ("angle_theta0", [float(lib.angle_types[k]["theta0"]) * DEG for k in self.angle_keys])):
            self.params[name] = Parameter(torch.tensor(vals, dtype=dt), requires_grad=name in train)
        register_periodic(self, "dihedral", [lib.dihedral_types[k]["terms"] for k in self.dihedral_keys], MAX_TERMS,
                          "dihedral_k" in train)
        register_periodic(self, "improper", [lib.improper_types[k]["terms"] for k in self.improper_keys],
                          MAX_IMPROPER_TERMS, "improper_k" in train)

    def type_index(self, name: str) -> int:
        if name not in self._type_index:
            raise KeyError(f"atom type {name!r} is not in library {self.name!r}")
        return self._type_index[name]

    def _resolve(self, kind, fn, *a) -> int:
        k = fn(self._tables[kind], *a)
        if k is None:
            raise KeyError(f"no {kind} type {'-'.join(a)} in library {self.name!r}")
        return self._index[kind][k]

    def resolve_bond(self, a, b):
        return self._resolve("bond", resolve_bond_type, a, b)

    def resolve_angle(self, a, b, c):
        return self._resolve("angle", resolve_angle_type, a, b, c)

    def resolve_dihedral(self, a, b, c, d):
        return self._resolve("dihedral", resolve_dihedral_type, a, b, c, d)

    def resolve_improper(self, *args):
        if len(args) == 1:
            if args[0] not in self._index["improper"]:
                raise KeyError(f"no improper type {args[0]!r} in library {self.name!r}")
            return self._index["improper"][args[0]]
        return self._resolve("improper", resolve_improper_type, *args)


@register_model("amber")
class Amber(FixedTopologyPotential):
    """An AMBER library bound to one topology (with its per-atom charges). Outputs ``e_bond``,
    ``e_angle``, ``e_torsion``, ``e_improper``, ``e_vdw``, ``e_coulomb``, ``e_vdw14``,
    ``e_coulomb14``, ``e_ref`` besides energies and ``charges``."""

    force_field_cls = None      # AmberForceField (set below the class)

    def __init__(self, ffield, topology, *, cutoff: float = 10.0, switch_width: float = 0.0,
                 charges: Optional[Sequence[float]] = None, fudge_lj: Optional[float] = None,
                 fudge_qq: Optional[float] = None, trainable=(), keep_intermediates: bool = False,
                 auto_impropers: bool = True, constrain_charge=True, use_fast="auto", atomic_energies=None):
        super().__init__()
        if isinstance(trainable, str):
            model_groups = set(MODEL_GROUPS) if trainable.lower() == "all" else ({trainable} & set(MODEL_GROUPS))
            groups = "all" if trainable.lower() == "all" else ((trainable,) if trainable not in MODEL_GROUPS else ())
        else:
            model_groups = {g for g in trainable if g in MODEL_GROUPS}
            groups = tuple(g for g in trainable if g not in MODEL_GROUPS)
        ffc = self.force_field_cls
        self.ff = ffield if isinstance(ffield, ffc) else ffc(ffield, trainable=groups)
        self.atom_ref = nn.Embedding(MAX_Z, 1)
        nn.init.zeros_(self.atom_ref.weight)
        self.atom_ref.weight.requires_grad_("atom_ref" in model_groups)
        self._train_charge = "charge" in model_groups
        self.auto_impropers = bool(auto_impropers)
        self.cutoff, self.switch_width = float(cutoff), float(switch_width)
        if not 0.0 <= self.switch_width < self.cutoff:
            raise ValueError("switch_width must satisfy 0 <= switch_width < cutoff")
        self.fudge_lj = self.ff.fudge_lj if fudge_lj is None else float(fudge_lj)
        self.fudge_qq = self.ff.fudge_qq if fudge_qq is None else float(fudge_qq)
        self.keep_intermediates, self.intermediates = bool(keep_intermediates), {}
        self.node_feature_dim = 1
        self.use_fast = resolve_use_fast(use_fast)
        top = topology if isinstance(topology, MolecularTopology) else read_topology(topology)
        self._bind(top)
        self._bind_charges(top, charges)
        self.species = sorted({int(z) for z in self.top_z.tolist()})
        if atomic_energies is not None:
            set_atomic_energies(self, atomic_energies)
        total = (float(self.charge.detach().sum()) if constrain_charge is True
                 else (None if constrain_charge is False else float(constrain_charge)))
        self.register_buffer("charge_total", torch.tensor(float("nan") if total is None else total,
                                                          dtype=self.charge.dtype), persistent=False)
        self._hold_total = total is not None      # a host flag: no device read per evaluation

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
            els = [SYMBOLS[int(ff.type_z[i])] if 0 < int(ff.type_z[i]) < len(SYMBOLS) else "X" for i in t]
            imps, keys = place_impropers(top, co, els, ff._tables["improper"])
            it = [ff.resolve_improper(k) for k in keys]
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

    def _bind_charges(self, top: MolecularTopology, charges) -> None:
        n = len(top.types)
        if charges is None:
            charges = top.charges if top.charges else [0.0] * n
        q = torch.as_tensor([float(c) for c in charges], dtype=torch.get_default_dtype())
        if q.numel() != n:
            raise ValueError(f"got {q.numel()} charges for {n} atoms")
        if self._train_charge:
            self.charge = Parameter(q)
        else:
            self.register_buffer("charge", q)

    @property
    def charges(self) -> Tensor:
        """Per-atom charges shifted uniformly onto the held total."""
        q = self.charge
        if not self._hold_total:
            return q
        return q - (q.sum() - self.charge_total) / q.shape[0]

    @staticmethod
    def _vdw_coulomb(rs_i, rs_j, eps_i, eps_j, q_i, q_j, r, r2):
        rstar = rs_i + rs_j
        x = (rstar * rstar / (r2 + TINY)) ** 3
        return geometric_mean(eps_i, eps_j) * (x * x - 2.0 * x), KE * q_i * q_j / r

    def forward(self, data: AtomicGraph) -> dict:
        N, B, n = self._check_batch(data)
        P, ff = self.ff.params, self.ff
        t = self.top_type.repeat(B)
        q = self.charges.repeat(B)
        bi, ai = batch_index(self.bond_index, n, B), batch_index(self.angle_index, n, B)
        di, ii = batch_index(self.dihedral_index, n, B), batch_index(self.improper_index, n, B)
        pi = batch_index(self.pair14_index, n, B)
        btype = self.bond_type.repeat(B)
        bv = pair_vectors(data, bi[0], bi[1])
        br = torch.sqrt((bv * bv).sum(1) + TINY)
        e_bond = P["bond_k"][btype] * (br - P["bond_r0"][btype]) ** 2
        e_bond_node = scatter_sum(0.5 * e_bond, bi[0], N) + scatter_sum(0.5 * e_bond, bi[1], N)
        atype = self.angle_type.repeat(B)
        theta = angle_theta(data, ai)
        e_angle = P["angle_k"][atype] * (theta - P["angle_theta0"][atype]) ** 2
        e_angle_node = scatter_sum(e_angle, ai[1], N)
        c, s = dihedral_cos_sin(data, di)
        e_tors = periodic_energy(ff, "dihedral", c, s, self.dihedral_type.repeat(B))
        e_tors_node = scatter_sum(e_tors, di[1], N)
        ci, si = dihedral_cos_sin(data, ii)
        e_impr = periodic_energy(ff, "improper", ci, si, self.improper_type.repeat(B))
        e_impr_node = scatter_sum(e_impr, ii[2], N)
        pv = pair_vectors(data, pi[0], pi[1])
        pr2 = (pv * pv).sum(1)
        pr = torch.sqrt(pr2 + TINY)
        ta, tb = t[pi[0]], t[pi[1]]
        v14, c14 = self._vdw_coulomb(P["rstar"][ta], P["rstar"][tb], P["epsilon"][ta], P["epsilon"][tb],
                                     q[pi[0]], q[pi[1]], pr, pr2)
        v14, c14 = self.fudge_lj * v14, self.fudge_qq * c14
        e_v14_node = scatter_sum(0.5 * v14, pi[0], N) + scatter_sum(0.5 * v14, pi[1], N)
        e_c14_node = scatter_sum(0.5 * c14, pi[0], N) + scatter_sum(0.5 * c14, pi[1], N)
        src, dst, _vec, r2, half, keep = self._pairs_once(data, self.excl_index, n)
        r = torch.sqrt(r2 + TINY)
        rs, ep = P["rstar"][t], P["epsilon"][t]
        vdw, coul = self._vdw_coulomb(rs[src], rs[dst], ep[src], ep[dst], q[src], q[dst], r, r2)
        w = keep.to(r.dtype) * half * quintic_switch(r, self.cutoff, self.switch_width)
        hv, hc = 0.5 * w * vdw, 0.5 * w * coul
        e_vdw_node = scatter_sum(hv, src, N) + scatter_sum(hv, dst, N)
        e_c_node = scatter_sum(hc, src, N) + scatter_sum(hc, dst, N)
        e_ref_node = self.atom_ref(data.atomic_numbers).squeeze(-1)
        node = (e_bond_node + e_angle_node + e_tors_node + e_impr_node + e_vdw_node + e_c_node + e_v14_node
                + e_c14_node + e_ref_node)
        if self.keep_intermediates:
            self.intermediates = dict(bond_r=br, e_bond=e_bond, angle_theta=theta, e_angle=e_angle, dihedral_cos=c,
                                      e_torsion=e_tors, improper_cos=ci, e_improper=e_impr, pair14_r=pr, e_vdw14=v14,
                                      e_coulomb14=c14, nb_r=r, nb_weight=w, nb_vdw=vdw, nb_coulomb=coul)
        agg = lambda x: self.aggregate_energy(x, data)  # noqa: E731
        return {"node_energy": node, "energy": agg(node), "charges": q, "node_features": q.unsqueeze(1),
                "e_bond": agg(e_bond_node), "e_angle": agg(e_angle_node), "e_torsion": agg(e_tors_node),
                "e_improper": agg(e_impr_node), "e_vdw": agg(e_vdw_node), "e_coulomb": agg(e_c_node),
                "e_vdw14": agg(e_v14_node), "e_coulomb14": agg(e_c14_node), "e_ref": agg(e_ref_node)}

    @classmethod
    def from_config(cls, cfg) -> "Amber":
        e = dict(cfg.extra or {})
        return cls(e.get("library", "ff94"), topology_from_options(e, "Amber"), cutoff=float(cfg.cutoff),
                   switch_width=float(e.get("switch_width") or 0.0), charges=_listy(e.get("charges")),
                   fudge_lj=_floaty(e, "fudge_lj"), fudge_qq=_floaty(e, "fudge_qq"),
                   trainable=_listy(e.get("trainable")) or (), constrain_charge=_constrain(e.get("constrain_charge", True)),
                   atomic_energies=e.get("atomic_energies"))


Amber.force_field_cls = AmberForceField
