"""CHARMM22 (MacKerell et al., J. Phys. Chem. B 102, 3586 (1998)): harmonic bonds, angles and
Urey-Bradley 1-3 terms, multi-term Fourier dihedrals, harmonic impropers ``K (psi - psi0)^2`` over
the atoms as listed (centre first), ``eps_ij [(Rmin_ij / r)^12 - 2 (Rmin_ij / r)^6]`` with
Lorentz-Berthelot mixing, per-type 1-4 Lennard-Jones parameters, pair overrides (NBFIX), unscaled
1-4 electrostatics and the CHARMM Coulomb constant 332.0716 kcal Å / (mol e^2). Bonded terms are
keyed by the atom types themselves. The CMAP cross term is not part of CHARMM22.

Library fields, the ``charmm22`` parameter set (``charmm22.frc``), improper resolution (exact in
either direction, then wildcard rows in table order) and improper placement from residue templates
(``-``/``+`` names for the neighbouring residues' atoms) follow the reference
(``src/xnn/ffnn/models/charmmlib.py``, ``charmm.py``).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence, Union

import torch
from torch import Tensor, nn
from torch.nn import Parameter, ParameterDict

from ..data import AtomicGraph
from ..data.elements import ATOMIC_NUMBERS, SYMBOLS
from ..models.registry import register_model
from ..ops.scatter import scatter_sum
from .amber import TWO_SIXTH, Amber, exact_trig, periodic_energy, register_periodic
from .frc import read_forcefield
from .geometry import TINY, angle_theta, batch_index, dihedral_cos_sin, geometric_mean, pair_vectors, quintic_switch
from .opls import (DEG, KCAL_TO_EV, WILDCARD, _constrain, _floaty, _groups, _listy, resolve_angle_type,
                   resolve_bond_type, resolve_dihedral_type, topology_from_options)
from .topology import MolecularTopology

COULOMB_CONSTANT = 332.0716
SCALE_14_COULOMB = 1.0
MAX_TERMS = 6
GROUPS = ("rstar", "epsilon", "rstar14", "epsilon14", "nbfix_rmin", "nbfix_eps", "bond_k", "bond_r0", "angle_k",
          "angle_theta0", "ub_k", "ub_s0", "dihedral_k", "improper_k")


@dataclass
class CharmmLibrary:
    """kcal/mol, Å, degrees. ``rstar`` = Rmin/2 with optional own 1-4 ``rstar14``/``epsilon14``;
    ``urey_bradley_types`` ``{"k", "s0"}``; torsions ``{"terms": [[K, n, delta], ...]}``; impropers
    ``{"k", "psi0"}``; ``nbfix_types`` ``{"rmin", "eps", "rmin14", "eps14"}`` per type pair."""
    atom_types: dict = field(default_factory=dict)
    bond_types: dict = field(default_factory=dict)
    angle_types: dict = field(default_factory=dict)
    urey_bradley_types: dict = field(default_factory=dict)
    dihedral_types: dict = field(default_factory=dict)
    improper_types: dict = field(default_factory=dict)
    nbfix_types: dict = field(default_factory=dict)
    coulomb_constant: float = COULOMB_CONSTANT
    scale_14_coulomb: float = SCALE_14_COULOMB
    name: str = "charmm"
    references: list = field(default_factory=list)
    templates: dict = field(default_factory=dict)
    fragments: dict = field(default_factory=dict)
    metadata: dict = field(default_factory=dict)
    notes: list = field(default_factory=list)

    def save(self, path: Union[str, Path]) -> None:
        keys = ("name", "references", "coulomb_constant", "scale_14_coulomb", "atom_types", "bond_types", "angle_types",
                "urey_bradley_types", "dihedral_types", "improper_types", "nbfix_types", "templates", "fragments",
                "metadata")
        Path(path).write_text(json.dumps({k: getattr(self, k) for k in keys}, indent=1, sort_keys=True) + "\n")


def resolve_improper_type(table: dict, i: str, j: str, k: str, l: str) -> Optional[str]:
    """Centre ``i``: the exact quadruple either way, then wildcard rows in table order (either way)."""
    quad = (i, j, k, l)
    for cand in (quad, quad[::-1]):
        if "-".join(cand) in table:
            return "-".join(cand)
    for key in table:
        pat = tuple(key.split("-"))
        if len(pat) == 4 and WILDCARD in pat and any(
                all(p == WILDCARD or p == q for p, q in zip(pat, cand)) for cand in (quad, quad[::-1])):
            return key
    return None


def place_impropers(top: MolecularTopology, fragments: dict, elements: Sequence[str]) -> list:
    """The impropers of the residue templates (centre first) mapped onto the topology; ``-X``/``+X``
    names pick the bonded atom of element ``X[0]`` outside the residue; impropers reaching past a
    chain end are dropped."""
    nbr: dict = {}
    for i, j in top.bonds:
        nbr.setdefault(i, []).append(j)
        nbr.setdefault(j, []).append(i)
    names, by_res, members = list(top.residue_names), {}, {}
    for atom, r in enumerate(top.residues):
        if r is None or r[0] >= len(names) or names[r[0]] not in fragments:
            continue
        atom_names = fragments[names[r[0]]].get("atom names", [])
        if r[1] < len(atom_names):
            by_res.setdefault(r[0], {})[str(atom_names[r[1]])] = atom
        members.setdefault(r[0], set()).add(atom)
    out = []
    for r in sorted(by_res):
        for quad in fragments[names[r]].get("impropers", []):
            if str(quad[0]) not in by_res[r]:
                continue
            center, atoms = by_res[r][str(quad[0])], []
            for nm in map(str, quad):
                if nm[0] in "+-":
                    cand = [a for a in nbr.get(center, []) if a not in members[r] and elements[a] == nm[1].upper()]
                    if len(cand) > 1:
                        raise ValueError(f"improper {quad} of residue {names[r]}: the reference {nm!r} matches "
                                         f"{len(cand)} atoms")
                    if not cand:
                        break
                    atoms.append(cand[0])
                elif nm in by_res[r]:
                    atoms.append(by_res[r][nm])
                else:
                    break
            if len(atoms) == 4:
                out.append(tuple(atoms))
    return out


_UNSUPPORTED = ("simple_fourier_angle", "tabulated_angle", "quartic_bond", "quartic_angle", "torsion_1", "torsion_3",
                "torsion_opls", "improper_opls", "improper_fourier", "buckingham", "nonbond(9-6)",
                "wilson_out_of_plane")


def _opt(values: dict, name: str) -> Optional[float]:
    v = values.get(name)
    return None if v is None or v == "" else float(v)


def from_forcefield(ff, strict: bool = True) -> CharmmLibrary:
    from .amber import _terms
    lib = CharmmLibrary(name=ff.name, metadata=dict(ff.metadata), templates=dict(ff.templates),
                        fragments=dict(ff.fragments), references=[r.text for r in ff.references_used()])
    lib.coulomb_constant = float(lib.metadata.get("coulomb_constant", COULOMB_CONSTANT))
    lib.scale_14_coulomb = float(lib.metadata.get("scale_14_coulomb", SCALE_14_COULOMB))
    extra = {k: len(ff.sections[k]) for k in ff.sections if k in _UNSUPPORTED}
    if extra:
        if strict:
            raise ValueError(f"force field {ff.name!r} uses functional forms the CHARMM model does not implement: "
                             f"{extra}. Pass strict=False to load it without those sections")
        lib.notes += [f"ignored section {k} ({n} rows)" for k, n in extra.items()]
    if "nonbond(12-6)" in ff.sections and ff.combination() != "arithmetic":
        raise ValueError(f"force field {ff.name!r} uses the {ff.combination()!r} combination rule; CHARMM requires "
                         "arithmetic (Lorentz-Berthelot)")
    rows14 = ff.rows("nonbond_1-4(12-6)")
    for name, at in ff.atom_types.items():
        e = {"element": ATOMIC_NUMBERS.get(str(at.get("El", "")), 0), "mass": float(at.get("Mass", 0.0)),
             "comment": str(at.get("Comment", ""))}
        try:
            e["connections"] = int(at.get("connections", 0))
        except (TypeError, ValueError):
            e["connections"] = 0
        lj = ff.nonbond(name) or (0.0, 0.0)
        e["rstar"], e["epsilon"] = float(lj[0]) * TWO_SIXTH / 2.0, float(lj[1])
        row = rows14.get((name,))
        if row is None:
            e["rstar14"] = e["epsilon14"] = None
        else:
            v = list(row.values.values())
            e["rstar14"], e["epsilon14"] = float(v[0]) * TWO_SIXTH / 2.0, float(v[1])
        lib.atom_types[name] = e

    def key(k):
        return "-".join(WILDCARD if x == "*" else x for x in k)
    for k, r in ff.rows("quadratic_bond").items():
        lib.bond_types[key(k)] = {"k": float(r.values["K2"]), "r0": float(r.values["R0"])}
    for k, r in ff.rows("quadratic_angle").items():
        lib.angle_types[key(k)] = {"k": float(r.values["K2"]), "theta0": float(r.values["Theta0"])}
    for k, r in ff.rows("urey_bradley").items():
        lib.urey_bradley_types[key(k)] = {"k": float(r.values["K2"]), "s0": float(r.values["S0"])}
    for k, r in ff.rows("torsion_fourier").items():
        lib.dihedral_types[key(k)] = {"terms": _terms(r.values, MAX_TERMS)}
    for k, r in ff.rows("improper_harmonic").items():
        lib.improper_types[key(k)] = {"k": float(r.values["K2"]), "psi0": float(r.values.get("Chi0", 0.0) or 0.0)}
    for k, r in ff.rows("nonbond_pair(12-6)").items():
        lib.nbfix_types[key(k)] = {"rmin": float(r.values["rmin"]), "eps": float(r.values["eps"]),
                                   "rmin14": _opt(r.values, "rmin14"), "eps14": _opt(r.values, "eps14")}
    return lib


def read_charmm(source: Union[str, Path], strict: bool = True) -> CharmmLibrary:
    s = str(source)
    if s.lower().endswith(".json"):
        d = json.loads(Path(s).read_text())
        lib = CharmmLibrary()
        for k, v in d.items():
            setattr(lib, k, v)
        return lib
    return from_forcefield(read_forcefield(s), strict=strict)


class CharmmForceField(nn.Module):
    def __init__(self, library: Union[CharmmLibrary, str, Path], trainable=()):
        super().__init__()
        lib = library if isinstance(library, CharmmLibrary) else read_charmm(str(library))
        dt = torch.get_default_dtype()
        train = _groups(trainable, GROUPS)
        self.name, self.coulomb_constant = lib.name, float(lib.coulomb_constant)
        self.fudge_lj, self.fudge_qq = 1.0, float(lib.scale_14_coulomb)
        self.type_names = list(lib.atom_types)
        self._type_index = {n: i for i, n in enumerate(self.type_names)}
        # CHARMM keys its bonded terms by the atom types themselves
        self.type_cls = self.type_cls_angle = self.type_cls_torsion = self.type_cls_oop = list(self.type_names)
        self.templates, self.fragments, self.metadata = dict(lib.templates), dict(lib.fragments), dict(lib.metadata)
        at = [lib.atom_types[n] for n in self.type_names]
        self.register_buffer("type_z", torch.tensor([int(a["element"]) for a in at], dtype=torch.long))
        self.register_buffer("type_mass", torch.tensor([float(a.get("mass", 0.0)) for a in at], dtype=dt))
        self._tables = {"bond": dict(lib.bond_types), "angle": dict(lib.angle_types),
                        "ub": dict(lib.urey_bradley_types), "dihedral": dict(lib.dihedral_types),
                        "improper": dict(lib.improper_types)}
        self.bond_keys, self.angle_keys, self.ub_keys = list(lib.bond_types), list(lib.angle_types), list(lib.urey_bradley_types)
        self.dihedral_keys, self.improper_keys = list(lib.dihedral_types), list(lib.improper_types)
        self.nbfix_keys = list(lib.nbfix_types)
        self._index = {t: {k: i for i, k in enumerate(getattr(self, f"{t}_keys"))}
                       for t in ("bond", "angle", "ub", "dihedral", "improper")}
        self.params = ParameterDict()

        def make(name, vals, grad=None):
            self.params[name] = Parameter(torch.tensor(vals, dtype=dt), requires_grad=(name in train) if grad is None else grad)
        own = [a.get("rstar14") is not None and a.get("epsilon14") is not None for a in at]
        self.register_buffer("own14", torch.tensor(own, dtype=torch.bool))
        make("rstar", [float(a["rstar"]) for a in at])
        make("epsilon", [float(a["epsilon"]) * KCAL_TO_EV for a in at])
        make("rstar14", [float(a["rstar14"]) if o else float(a["rstar"]) for a, o in zip(at, own)])
        make("epsilon14", [(float(a["epsilon14"]) if o else float(a["epsilon"])) * KCAL_TO_EV for a, o in zip(at, own)])
        pairs = [k.split("-") for k in self.nbfix_keys]
        self.register_buffer("nbfix_i", torch.tensor([self.type_index(a) for a, _ in pairs], dtype=torch.long))
        self.register_buffer("nbfix_j", torch.tensor([self.type_index(b) for _, b in pairs], dtype=torch.long))
        rows = [lib.nbfix_types[k] for k in self.nbfix_keys]
        make("nbfix_rmin", [float(r["rmin"]) for r in rows])
        make("nbfix_eps", [float(r["eps"]) * KCAL_TO_EV for r in rows])
        make("nbfix_rmin14", [float(r["rmin"] if r.get("rmin14") is None else r["rmin14"]) for r in rows],
             "nbfix_rmin" in train)
        make("nbfix_eps14", [float(r["eps"] if r.get("eps14") is None else r["eps14"]) * KCAL_TO_EV for r in rows],
             "nbfix_eps" in train)
        make("bond_k", [float(lib.bond_types[k]["k"]) * KCAL_TO_EV for k in self.bond_keys])
        make("bond_r0", [float(lib.bond_types[k]["r0"]) for k in self.bond_keys])
        make("angle_k", [float(lib.angle_types[k]["k"]) * KCAL_TO_EV for k in self.angle_keys])
        make("angle_theta0", [float(lib.angle_types[k]["theta0"]) * DEG for k in self.angle_keys])
        make("ub_k", [float(lib.urey_bradley_types[k]["k"]) * KCAL_TO_EV for k in self.ub_keys])
        make("ub_s0", [float(lib.urey_bradley_types[k]["s0"]) for k in self.ub_keys])
        register_periodic(self, "dihedral", [lib.dihedral_types[k]["terms"] for k in self.dihedral_keys], MAX_TERMS,
                          "dihedral_k" in train)
        make("improper_k", [float(lib.improper_types[k]["k"]) * KCAL_TO_EV for k in self.improper_keys])
        c, s = exact_trig(torch.tensor([float(lib.improper_types[k].get("psi0", 0.0)) * DEG for k in self.improper_keys],
                                       dtype=torch.float64))
        self.register_buffer("improper_cos", c.to(dt))
        self.register_buffer("improper_sin", s.to(dt))

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

    def resolve_urey_bradley(self, a, b, c) -> Optional[int]:
        k = resolve_angle_type(self._tables["ub"], a, b, c)
        return None if k is None else self._index["ub"][k]

    def resolve_dihedral(self, a, b, c, d):
        return self._resolve("dihedral", resolve_dihedral_type, a, b, c, d)

    def resolve_improper(self, *args):
        if len(args) == 1:
            key = args[0]
            if key not in self._index["improper"]:
                key = "-".join(key.split("-")[::-1])
                if key not in self._index["improper"]:
                    raise KeyError(f"no improper type {args[0]!r} in library {self.name!r}")
            return self._index["improper"][key]
        return self._resolve("improper", resolve_improper_type, *args)

    def pair_tables(self):
        """``(T, T)`` ``rmin``, ``eps`` and their 1-4 versions: Lorentz-Berthelot of the per-type values
        (own 1-4 values where a type has them) with the NBFIX pairs written over."""
        P = self.params
        rs, eps = P["rstar"], P["epsilon"]
        rs14, eps14 = torch.where(self.own14, P["rstar14"], rs), torch.where(self.own14, P["epsilon14"], eps)
        out = []
        for r, e, pr, pe in ((rs, eps, P["nbfix_rmin"], P["nbfix_eps"]),
                             (rs14, eps14, P["nbfix_rmin14"], P["nbfix_eps14"])):
            rmin = r[:, None] + r[None, :]
            well = geometric_mean(e[:, None].expand_as(rmin), e[None, :].expand_as(rmin))
            if self.nbfix_i.numel():
                ii, jj = torch.cat([self.nbfix_i, self.nbfix_j]), torch.cat([self.nbfix_j, self.nbfix_i])
                rmin = rmin.index_put((ii, jj), torch.cat([pr, pr]))
                well = well.index_put((ii, jj), torch.cat([pe, pe]))
            out += [rmin, well]
        return tuple(out)


@register_model("charmm")
class Charmm(Amber):
    """A CHARMM library bound to one topology with its per-atom charges. Outputs ``e_bond``,
    ``e_angle``, ``e_urey_bradley``, ``e_torsion``, ``e_improper``, ``e_vdw``, ``e_coulomb``,
    ``e_vdw14``, ``e_coulomb14``, ``e_ref``."""

    force_field_cls = CharmmForceField

    def __init__(self, ffield, topology, *, coulomb_constant: Optional[float] = None, **kw):
        super().__init__(ffield, topology, **kw)
        self.coulomb_constant = self.ff.coulomb_constant if coulomb_constant is None else float(coulomb_constant)

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
        nm = [ff.type_names[i] for i in t]
        bt = [get(ff.resolve_bond, nm[i], nm[j]) for i, j in top.bonds]
        at = [get(ff.resolve_angle, nm[i], nm[j], nm[k]) for i, j, k in top.angles]
        ub_pairs, ub_type = [], []
        for i, j, k in top.angles:
            row = ff.resolve_urey_bradley(nm[i], nm[j], nm[k])
            if row is not None:
                ub_pairs.append((i, k))
                ub_type.append(row)
        dt = [get(ff.resolve_dihedral, nm[i], nm[j], nm[k], nm[l]) for i, j, k, l in top.dihedrals]
        imps = [tuple(int(x) for x in im) for im in top.impropers]
        if top.improper_keys:
            it = [get(ff.resolve_improper, k) for k in top.improper_keys]
        elif imps:
            it = [get(ff.resolve_improper, nm[i], nm[j], nm[k], nm[l]) for i, j, k, l in imps]
        elif self.auto_impropers and top.residues:
            els = [SYMBOLS[int(ff.type_z[i])] if 0 < int(ff.type_z[i]) < len(SYMBOLS) else "X" for i in t]
            imps = place_impropers(top, ff.fragments, els)
            it = [get(ff.resolve_improper, nm[i], nm[j], nm[k], nm[l]) for i, j, k, l in imps]
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
        self._buf("ub_index", ub_pairs, 2)
        self._buf("ub_type", ub_type, 1)
        self._buf("dihedral_index", top.dihedrals, 4)
        self._buf("dihedral_type", dt, 1)
        self.impropers = imps
        self._buf("improper_index", imps, 4)
        self._buf("improper_type", it, 1)
        self._buf("pair14_index", top.pairs14, 2)
        self._buf("excl_index", sorted(set(top.exclusions) | set(top.pairs14)), 2)

    @staticmethod
    def _lj(rmin: Tensor, eps: Tensor, r2: Tensor) -> Tensor:
        x = (rmin * rmin / (r2 + TINY)) ** 3
        return eps * (x * x - 2.0 * x)

    def forward(self, data: AtomicGraph) -> dict:
        N, B, n = self._check_batch(data)
        P, ff = self.ff.params, self.ff
        t = self.top_type.repeat(B)
        q = self.charges.repeat(B)
        ke = self.coulomb_constant * KCAL_TO_EV
        rmin_t, eps_t, rmin14_t, eps14_t = ff.pair_tables()
        bi, ai, ui = (batch_index(x, n, B) for x in (self.bond_index, self.angle_index, self.ub_index))
        di, ii, pi = (batch_index(x, n, B) for x in (self.dihedral_index, self.improper_index, self.pair14_index))
        btype = self.bond_type.repeat(B)
        bv = pair_vectors(data, bi[0], bi[1])
        br = torch.sqrt((bv * bv).sum(1) + TINY)
        e_bond = P["bond_k"][btype] * (br - P["bond_r0"][btype]) ** 2
        e_bond_node = scatter_sum(0.5 * e_bond, bi[0], N) + scatter_sum(0.5 * e_bond, bi[1], N)
        atype = self.angle_type.repeat(B)
        theta = angle_theta(data, ai)
        e_angle = P["angle_k"][atype] * (theta - P["angle_theta0"][atype]) ** 2
        e_angle_node = scatter_sum(e_angle, ai[1], N)
        utype = self.ub_type.repeat(B)
        uv = pair_vectors(data, ui[0], ui[1])
        ur = torch.sqrt((uv * uv).sum(1) + TINY)
        e_ub = P["ub_k"][utype] * (ur - P["ub_s0"][utype]) ** 2
        e_ub_node = scatter_sum(0.5 * e_ub, ui[0], N) + scatter_sum(0.5 * e_ub, ui[1], N)
        c1, s1 = dihedral_cos_sin(data, di)
        e_tors = periodic_energy(ff, "dihedral", c1, s1, self.dihedral_type.repeat(B))
        e_tors_node = scatter_sum(e_tors, di[1], N)
        itype = self.improper_type.repeat(B)
        ci, si = dihedral_cos_sin(data, ii)
        c0, s0 = ff.improper_cos[itype], ff.improper_sin[itype]
        dphi = torch.atan2(si * c0 - ci * s0, ci * c0 + si * s0)
        e_impr = P["improper_k"][itype] * dphi * dphi
        e_impr_node = scatter_sum(e_impr, ii[0], N)
        src, dst, _vec, r2, half, keep = self._pairs_once(data, self.excl_index, n)
        r = torch.sqrt(r2 + TINY)
        ts, td = t[src], t[dst]
        vdw = self._lj(rmin_t[ts, td], eps_t[ts, td], r2)
        coul = ke * q[src] * q[dst] / r
        w = keep.to(r.dtype) * half * quintic_switch(r, self.cutoff, self.switch_width)
        hv, hc = 0.5 * w * vdw, 0.5 * w * coul
        e_vdw_node = scatter_sum(hv, src, N) + scatter_sum(hv, dst, N)
        e_c_node = scatter_sum(hc, src, N) + scatter_sum(hc, dst, N)
        p0, p1 = t[pi[0]], t[pi[1]]
        pv = pair_vectors(data, pi[0], pi[1])
        pr2 = (pv * pv).sum(1)
        pr = torch.sqrt(pr2 + TINY)
        v14 = self._lj(rmin14_t[p0, p1], eps14_t[p0, p1], pr2)
        c14 = self.fudge_qq * ke * q[pi[0]] * q[pi[1]] / pr
        e_v14_node = scatter_sum(0.5 * v14, pi[0], N) + scatter_sum(0.5 * v14, pi[1], N)
        e_c14_node = scatter_sum(0.5 * c14, pi[0], N) + scatter_sum(0.5 * c14, pi[1], N)
        e_ref_node = self.atom_ref(data.atomic_numbers).squeeze(-1)
        node = (e_bond_node + e_angle_node + e_ub_node + e_tors_node + e_impr_node + e_vdw_node + e_c_node
                + e_v14_node + e_c14_node + e_ref_node)
        if self.keep_intermediates:
            self.intermediates = dict(bond_r=br, e_bond=e_bond, angle_theta=theta, e_angle=e_angle, ub_r=ur,
                                      e_urey_bradley=e_ub, dihedral_cos=c1, dihedral_sin=s1, e_torsion=e_tors,
                                      improper_dphi=dphi, e_improper=e_impr, pair14_r=pr, e_vdw14=v14, e_coulomb14=c14)
        agg = lambda x: self.aggregate_energy(x, data)  # noqa: E731
        return {"node_energy": node, "energy": agg(node), "charges": q, "node_features": q.unsqueeze(1),
                "e_bond": agg(e_bond_node), "e_angle": agg(e_angle_node), "e_urey_bradley": agg(e_ub_node),
                "e_torsion": agg(e_tors_node), "e_improper": agg(e_impr_node), "e_vdw": agg(e_vdw_node),
                "e_coulomb": agg(e_c_node), "e_vdw14": agg(e_v14_node), "e_coulomb14": agg(e_c14_node),
                "e_ref": agg(e_ref_node)}

    @classmethod
    def from_config(cls, cfg) -> "Charmm":
        e = dict(cfg.extra or {})
        return cls(e.get("library", "charmm22"), topology_from_options(e, "Charmm"), cutoff=float(cfg.cutoff),
                   switch_width=float(e.get("switch_width") or 0.0), charges=_listy(e.get("charges")),
                   coulomb_constant=_floaty(e, "coulomb_constant"), trainable=_listy(e.get("trainable")) or (),
                   constrain_charge=_constrain(e.get("constrain_charge", True)),
                   atomic_energies=e.get("atomic_energies"))
