"""LAMMPS inputs (a data file and the input commands) for the fixed-topology force fields, so a
model with trained parameters can be run or cross-checked in LAMMPS (``units real``,
``atom_style full``).

Styles per force field:

* OPLS: ``lj/cut/coul/cut`` with geometric mixing, harmonic bonds and angles, ``dihedral_style
  opls`` (the series constants ``V0``, which LAMMPS has no term for, come back as an energy
  offset) and ``improper_style cvff``;
* AMBER: arithmetic mixing, ``dihedral_style fourier`` (each torsion's non-zero terms with their
  phases) and ``improper_style cvff``;
* CHARMM: ``lj/charmm/coul/charmm`` with the full pair table written per type pair (NBFIX and the
  1-4 values included), Urey-Bradley terms in ``angle_style charmm``, ``dihedral_style charmm``
  carrying the 1-4 pairs (weight ``1/count`` for a pair closing several dihedrals, 0 for pairs
  that are not 1-4), harmonic impropers;
* DREIDING: ``lj/cut`` or ``buck`` (exp-6), Morse or harmonic bonds scaled by bond order,
  ``cosine/squared`` angles (``cosine`` at linear centres), ``dihedral_style harmonic``,
  ``improper_style umbrella`` and ``hbond/dreiding/lj`` overlaid for hydrogen bonds.

Charges are rescaled so that LAMMPS's Coulomb constant (332.06371) gives the model's Coulomb
energies. Bonded types are the distinct parameter sets, numbered in order of first use. The
file layout, command order and number formats are those the reference writes
(``src/xnn/ffnn/models/lammps_input.py``), so that inputs from either side are interchangeable.
Cells must be orthorhombic; a cluster gets a shrink-wrapped box padded by the cutoff.

Design: every writer fills a :class:`_Deck` -- atoms, one :class:`_Kinds` table per bonded section
(parameter key -> type id) with its member rows, the style lines and the coefficient lines -- and
the deck renders the two texts.
"""
from __future__ import annotations

import math
from pathlib import Path
from typing import Callable, Dict, List, Optional, Sequence, Tuple, Union

import numpy as np

LAMMPS_COULOMB = 332.06371
_DEG = math.pi / 180.0
#: bonded sections in file order: (style keyword, data-file header)
_KINDS = (("bond", "Bonds"), ("angle", "Angles"), ("dihedral", "Dihedrals"), ("improper", "Impropers"))
_ROOT6_2 = 2.0 ** (1.0 / 6.0)


def _q(x, nd: int = 14) -> float:
    """Parameter value as stored in a type key (rounded so equal parameters share one type)."""
    return round(float(x), nd)


def _g15(x) -> str:
    return f"{x:.15g}"


class _Kinds:
    """Distinct parameter keys of one bonded section, numbered from 1 by first use, plus the
    section's rows ``(type id, atom ids...)``."""

    def __init__(self):
        self.ids: Dict[tuple, int] = {}
        self.rows: List[Tuple[int, ...]] = []

    def add(self, key: tuple, atoms: Sequence[int]) -> None:
        tid = self.ids.get(key)
        if tid is None:
            tid = self.ids[key] = len(self.ids) + 1
        self.rows.append((tid, *[int(a) + 1 for a in atoms]))

    def items(self):
        return ((tid, key) for key, tid in self.ids.items())


class _Deck:
    def __init__(self, title: str, cutoff: float):
        self.title = title
        self.cutoff = float(cutoff)
        self.kinds = {k: _Kinds() for k, _ in _KINDS}
        self.type_of: Dict[object, int] = {}     # atom type label -> LAMMPS atom type id
        self.masses: Dict[int, float] = {}
        self.atoms: List[int] = []
        self.charges: np.ndarray = np.zeros(0)
        self.head: List[str] = []                # commands before read_data
        self.coeffs: List[str] = []              # commands after read_data
        self.offset = 0.0

    def atom_types(self, labels: Sequence, mass: Callable[[object], float]) -> None:
        for lab in labels:
            if lab not in self.type_of:
                tid = self.type_of[lab] = len(self.type_of) + 1
                self.masses[tid] = mass(lab)
        self.atoms = [self.type_of[lab] for lab in labels]

    def used_styles(self, styles: Dict[str, str]) -> List[str]:
        return [f"{k}_style {styles[k]}" for k, _ in _KINDS if self.kinds[k].rows]

    def data_text(self, pos: np.ndarray, bounds: np.ndarray) -> str:
        k = self.kinds
        out = [self.title, "", f"{len(self.atoms)} atoms"]
        out += [f"{len(k[name].rows)} {header.lower()}" for name, header in _KINDS]
        out += ["", f"{len(self.masses)} atom types"]
        out += [f"{len(k[name].ids)} {name} types" for name, _ in _KINDS]
        out.append("")
        for axis, x in enumerate("xyz"):
            out.append(f"{float(bounds[axis, 0])!r} {float(bounds[axis, 1])!r} {x}lo {x}hi")
        out += ["", "Masses", ""] + [f"{tid} {m:.6f}" for tid, m in self.masses.items()]
        out += ["", "Atoms # full", ""]
        for n, (tid, q, r) in enumerate(zip(self.atoms, self.charges, pos), start=1):
            out.append(f"{n} 1 {tid} {q:.15g} {r[0]:.14f} {r[1]:.14f} {r[2]:.14f}")
        for name, header in _KINDS:
            rows = k[name].rows
            if rows:
                out += ["", header, ""]
                out += [" ".join(map(str, (n, *row))) for n, row in enumerate(rows, start=1)]
        return "\n".join(out) + "\n"

    def commands(self) -> List[str]:
        return self.head + ["read_data DATAFILE"] + self.coeffs


def _base_head(boundary: str) -> List[str]:
    return ["units real", "atom_style full", f"boundary {boundary}"]


def _host(params) -> Dict[str, "np.ndarray"]:
    return {k: v.detach().double().cpu() for k, v in params.items()}


def _phase_deg(sin, cos) -> float:
    return math.degrees(math.atan2(float(sin), float(cos)))


# ----------------------------------------------------------------------------- OPLS
def _opls(model, boundary: str) -> _Deck:
    from .opls import KCAL_TO_EV, KE
    to_kcal = 1.0 / KCAL_TO_EV
    ff, P = model.ff, _host(model.ff.params)
    deck = _Deck("xnn OPLS", model.cutoff)
    labels = model.top_type.tolist()
    deck.atom_types(labels, lambda t: float(ff.type_mass[t]))
    deck.charges = (ff.charges.detach().double().cpu()[model.top_type.cpu()].numpy()
                    * math.sqrt(KE * to_kcal / LAMMPS_COULOMB))
    spec = {
        "bond": (model.bond_index, model.bond_type,
                 lambda t: (_q(P["bond_k"][t] * to_kcal), _q(P["bond_r0"][t]))),
        "angle": (model.angle_index, model.angle_type,
                  lambda t: (_q(P["angle_k"][t] * to_kcal), _q(P["angle_theta0"][t] / _DEG))),
        "dihedral": (model.dihedral_index, model.dihedral_type,
                     lambda t: tuple(_q(P["dihedral_v"][t, s] * to_kcal) for s in range(1, 5))),
        "improper": (model.improper_index, model.improper_type,
                     lambda t: (_q(0.5 * P["improper_v2"][t] * to_kcal),)),
    }
    for name, (index, types, key) in spec.items():
        idx = index.t().tolist()
        for atoms, t in zip(idx, types.tolist()):
            deck.kinds[name].add(key(int(t)), atoms)
    deck.offset = float(P["dihedral_v"][model.dihedral_type.cpu(), 0].sum()) * to_kcal
    deck.head = _base_head(boundary) + [
        f"pair_style lj/cut/coul/cut {deck.cutoff!r}", "pair_modify mix geometric",
        f"special_bonds lj 0.0 0.0 {model.fudge_lj!r} coul 0.0 0.0 {model.fudge_qq!r}",
    ] + deck.used_styles({"bond": "harmonic", "angle": "harmonic", "dihedral": "opls", "improper": "cvff"})
    for lab, tid in deck.type_of.items():
        deck.coeffs.append(f"pair_coeff {tid} {tid} {_g15(float(P['epsilon'][lab]) * to_kcal)} "
                           f"{_g15(float(P['sigma'][lab]))}")
    k = deck.kinds
    deck.coeffs += [f"bond_coeff {t} {_g15(a)} {_g15(b)}" for t, (a, b) in k["bond"].items()]
    deck.coeffs += [f"angle_coeff {t} {_g15(a)} {_g15(b)}" for t, (a, b) in k["angle"].items()]
    deck.coeffs += [f"dihedral_coeff {t} " + " ".join(map(_g15, key)) for t, key in k["dihedral"].items()]
    deck.coeffs += [f"improper_coeff {t} {_g15(key[0])} -1 2" for t, key in k["improper"].items()]
    return deck


# ----------------------------------------------------------------------------- AMBER
def _amber(model, boundary: str) -> _Deck:
    from .amber import KCAL_TO_EV, KE_KCAL
    to_kcal = 1.0 / KCAL_TO_EV
    ff, top, P = model.ff, model.topology, _host(model.ff.params)
    deck = _Deck("xnn AMBER", model.cutoff)
    tindex = {t: ff.type_index(t) for t in dict.fromkeys(top.types)}
    deck.atom_types(top.types, lambda t: float(ff.type_mass[tindex[t]]))
    deck.charges = model.charges.detach().double().cpu().numpy() * math.sqrt(KE_KCAL / LAMMPS_COULOMB)
    k = deck.kinds
    for atoms, t in zip(top.bonds, model.bond_type.tolist()):
        k["bond"].add((_q(P["bond_k"][t] * to_kcal), _q(P["bond_r0"][t])), atoms)
    for atoms, t in zip(top.angles, model.angle_type.tolist()):
        k["angle"].add((_q(P["angle_k"][t] * to_kcal), _q(P["angle_theta0"][t] / _DEG)), atoms)
    n_terms = P["dihedral_k"].shape[1]
    for atoms, t in zip(top.dihedrals, model.dihedral_type.tolist()):
        series = []
        for s in range(n_terms):
            amp = float(P["dihedral_k"][t, s])
            if amp != 0.0:
                series.append((_q(amp * to_kcal), int(ff.dihedral_n[t, s]),
                               _q(_phase_deg(ff.dihedral_sin[t, s], ff.dihedral_cos[t, s]))))
        if series:
            k["dihedral"].add(tuple(series), atoms)
    for atoms, t in zip(model.impropers, model.improper_type.tolist()):
        k["improper"].add((_q(P["improper_k"][t, 0] * to_kcal), int(round(float(ff.improper_cos[t, 0]))),
                           int(ff.improper_n[t, 0])), atoms)
    deck.head = _base_head(boundary) + [
        f"pair_style lj/cut/coul/cut {deck.cutoff!r}", "pair_modify mix arithmetic",
        f"special_bonds lj 0.0 0.0 {model.fudge_lj!r} coul 0.0 0.0 {model.fudge_qq!r}",
    ] + deck.used_styles({"bond": "harmonic", "angle": "harmonic", "dihedral": "fourier", "improper": "cvff"})
    rstar_to_sigma = 2.0 / _ROOT6_2
    for lab, tid in deck.type_of.items():
        x = tindex[lab]
        deck.coeffs.append(f"pair_coeff {tid} {tid} {_g15(float(P['epsilon'][x]) * to_kcal)} "
                           f"{_g15(float(P['rstar'][x]) * rstar_to_sigma)}")
    deck.coeffs += [f"bond_coeff {t} {_g15(a)} {_g15(b)}" for t, (a, b) in k["bond"].items()]
    deck.coeffs += [f"angle_coeff {t} {_g15(a)} {_g15(b)}" for t, (a, b) in k["angle"].items()]
    for t, series in k["dihedral"].items():
        deck.coeffs.append(f"dihedral_coeff {t} {len(series)} "
                           + " ".join(f"{_g15(a)} {n} {_g15(d)}" for a, n, d in series))
    deck.coeffs += [f"improper_coeff {t} {_g15(a)} {s} {n}" for t, (a, s, n) in k["improper"].items()]
    return deck


# ----------------------------------------------------------------------------- CHARMM
def _charmm(model, boundary: str) -> _Deck:
    from .charmm import KCAL_TO_EV
    to_kcal = 1.0 / KCAL_TO_EV
    ff, top, P = model.ff, model.topology, _host(model.ff.params)
    deck = _Deck("xnn CHARMM", model.cutoff)
    tindex = {t: ff.type_index(t) for t in dict.fromkeys(top.types)}
    deck.atom_types(top.types, lambda t: float(ff.type_mass[tindex[t]]))
    deck.charges = (model.charges.detach().double().cpu().numpy()
                    * math.sqrt(float(model.coulomb_constant) / LAMMPS_COULOMB))
    rmin, eps, rmin14, eps14 = (x.detach().double().cpu() for x in ff.pair_tables())
    k = deck.kinds
    for atoms, t in zip(top.bonds, model.bond_type.tolist()):
        k["bond"].add((_q(P["bond_k"][t] * to_kcal), _q(P["bond_r0"][t])), atoms)
    urey = {}
    for (a, c), t in zip(model.ub_index.t().tolist(), model.ub_type.tolist()):
        urey[(a, c)] = (_q(P["ub_k"][t] * to_kcal), _q(P["ub_s0"][t]))
    for atoms, t in zip(top.angles, model.angle_type.tolist()):
        ends = (atoms[0], atoms[2])
        k["angle"].add((_q(P["angle_k"][t] * to_kcal), _q(P["angle_theta0"][t] / _DEG)) + urey.get(ends, (0.0, 0.0)),
                       atoms)
    # dihedral_style charmm also applies the 1-4 pairs: weight 1/count for a pair at the ends of
    # several dihedrals, 0 when the ends are not a 1-4 pair (rings)
    pairs14 = {tuple(p) for p in top.pairs14}
    ends_count: Dict[Tuple[int, int], int] = {}
    for d in top.dihedrals:
        e = tuple(sorted((d[0], d[3])))
        ends_count[e] = ends_count.get(e, 0) + 1
    n_terms = P["dihedral_k"].shape[1]
    for atoms, t in zip(top.dihedrals, model.dihedral_type.tolist()):
        e = tuple(sorted((atoms[0], atoms[3])))
        w14 = 1.0 / ends_count[e] if e in pairs14 else 0.0
        for s in range(n_terms):
            if float(ff.dihedral_mask[t, s]) == 0.0:
                continue
            phase = int(round(_phase_deg(ff.dihedral_sin[t, s], ff.dihedral_cos[t, s]))) % 360
            k["dihedral"].add((_q(P["dihedral_k"][t, s] * to_kcal), int(ff.dihedral_n[t, s]), phase,
                               w14 if s == 0 else 0.0), atoms)
    for atoms, t in zip(model.impropers, model.improper_type.tolist()):
        k["improper"].add((_q(P["improper_k"][t] * to_kcal), _q(_phase_deg(ff.improper_sin[t], ff.improper_cos[t]))),
                          atoms)
    rc = deck.cutoff
    deck.head = _base_head(boundary) + [f"pair_style lj/charmm/coul/charmm {rc - 1e-6!r} {rc!r}",
                                        "special_bonds charmm"]
    deck.head += deck.used_styles({"bond": "harmonic", "angle": "charmm", "dihedral": "charmm",
                                   "improper": "harmonic"})
    labs = list(deck.type_of)
    for ia, a in enumerate(labs):
        for b in labs[ia:]:
            x, y = tindex[a], tindex[b]
            deck.coeffs.append(
                f"pair_coeff {deck.type_of[a]} {deck.type_of[b]} {_g15(float(eps[x, y]) * to_kcal)} "
                f"{_g15(float(rmin[x, y]) / _ROOT6_2)} {_g15(float(eps14[x, y]) * to_kcal)} "
                f"{_g15(float(rmin14[x, y]) / _ROOT6_2)}")
    deck.coeffs += [f"bond_coeff {t} {_g15(a)} {_g15(b)}" for t, (a, b) in k["bond"].items()]
    deck.coeffs += [f"angle_coeff {t} " + " ".join(map(_g15, key)) for t, key in k["angle"].items()]
    deck.coeffs += [f"dihedral_coeff {t} {_g15(a)} {n} {ph} {_g15(w)}" for t, (a, n, ph, w) in k["dihedral"].items()]
    deck.coeffs += [f"improper_coeff {t} {_g15(a)} {_g15(b)}" for t, (a, b) in k["improper"].items()]
    return deck


# ----------------------------------------------------------------------------- DREIDING
def _dreiding_pair_args(ff, P, x: int, y: int, to_kcal: float) -> str:
    if ff.form == "x6":
        # exp-6 as buck: A exp(-r / rho) - C / r^6; A and C combine geometrically, 1/rho arithmetically
        zeta = [max(float(P["x6_zeta"][i]), 6.0 + 1e-6) for i in (x, y)]
        r0 = [float(P["vdw_r0"][i]) for i in (x, y)]
        d0 = [float(P["vdw_d0"][i]) * to_kcal for i in (x, y)]
        A = [d * 6.0 / (zt - 6.0) * math.exp(zt) for d, zt in zip(d0, zeta)]
        Cc = [d * zt / (zt - 6.0) * r ** 6 for d, zt, r in zip(d0, zeta, r0)]
        rho = 1.0 / (0.5 * (zeta[0] / r0[0] + zeta[1] / r0[1]))
        return f"{math.sqrt(A[0] * A[1]):.14g} {rho:.14g} {math.sqrt(Cc[0] * Cc[1]):.14g}"
    d0 = math.sqrt(float(P["vdw_d0"][x] * P["vdw_d0"][y])) * to_kcal
    ra, rb = float(P["vdw_r0"][x]), float(P["vdw_r0"][y])
    r0 = math.sqrt(ra * rb) if ff.combination == "geometric" else 0.5 * (ra + rb)
    return f"{d0:.14g} {r0 / _ROOT6_2:.14g}"


def _dreiding(model, boundary: str) -> _Deck:
    from .dreiding import KCAL_TO_EV, KE
    to_kcal = 1.0 / KCAL_TO_EV
    ff, top, P = model.ff, model.topology, _host(model.ff.params)
    deck = _Deck("xnn DREIDING", model.cutoff)
    tindex = {t: ff.type_index(t) for t in dict.fromkeys(top.types)}
    deck.atom_types(top.types, lambda t: float(ff.type_mass[tindex[t]]) or 1.0)
    n = len(top.types)
    deck.charges = (model.charge.detach().double().cpu().numpy() * math.sqrt(KE * to_kcal / LAMMPS_COULOMB)
                    if model.has_coulomb else np.zeros(n))
    k = deck.kinds
    morse = model.bond_style == "morse"
    orders = list(top.bond_orders) or [1.0] * len(top.bonds)
    radius = lambda a: float(P["radius"][tindex[top.types[a]]])  # noqa: E731
    for (i, j), order in zip(top.bonds, orders):
        r0 = radius(i) + radius(j) - ff.delta
        kb = order * float(P["bond_k"])
        if morse:
            de = order * float(P["bond_d"])
            k["bond"].add((_q(de * to_kcal), _q(math.sqrt(kb / (2.0 * de))), _q(r0)), (i, j))
        else:
            k["bond"].add((_q(0.5 * kb * to_kcal), _q(r0)), (i, j))
    ka = float(P["angle_k"]) * to_kcal
    for (i, j, l), linear in zip(top.angles, model.angle_linear.tolist()):
        th0 = float(P["theta0"][tindex[top.types[j]]])
        key = ("cosine", _q(ka), 0.0) if linear else \
            ("cosine/squared", _q(0.5 * ka / math.sin(th0) ** 2), _q(th0 / _DEG))
        k["angle"].add(key, (i, j, l))
    for atoms, rule, wt in zip(model.dihedral_index.t().tolist(), model.dihedral_rule.tolist(),
                               model.dihedral_weight.tolist()):
        v = float(wt) * float(P["torsion_v"][rule]) * to_kcal
        k["dihedral"].add((_q(0.5 * v), -int(ff.rule_sign[rule]), int(ff.rule_n[rule])), atoms)
    for atoms in model.inversion_index.t().tolist():
        x = tindex[top.types[atoms[0]]]
        k["improper"].add((_q(float(P["oop_k"][x]) * to_kcal / 3.0), _q(float(P["oop_psi0"][x]) / _DEG)), atoms)
    hyd = model.hbond_hydrogens.cpu()
    with_hb = model.use_hbond and bool((hyd >= 0).any())
    vdw = "buck" if ff.form == "x6" else "lj/cut"
    base = f"{vdw}{'/coul/cut' if model.has_coulomb else ''} {deck.cutoff!r}"
    hb_angle = math.acos(model.hbond_cos) / _DEG
    hb_tail = f"{model.hbond_cutoff!r} {model.hbond_cutoff!r} {hb_angle!r}"
    deck.head = _base_head(boundary) + ["special_bonds lj/coul 0.0 0.0 1.0"]
    deck.head.append(f"pair_style hybrid/overlay {base} hbond/dreiding/lj 4 {hb_tail}" if with_hb
                     else f"pair_style {base}")
    angle_styles = sorted({key[0] for key in k["angle"].ids})
    if k["bond"].ids:
        deck.head.append(f"bond_style {'morse' if morse else 'harmonic'}")
    if k["angle"].ids:
        deck.head.append("angle_style " + (f"hybrid {' '.join(angle_styles)}" if len(angle_styles) > 1
                                           else angle_styles[0]))
    if k["dihedral"].ids:
        deck.head.append("dihedral_style harmonic")
    if k["improper"].ids:
        deck.head.append("improper_style umbrella")
    prefix = f"{base.split()[0]} " if with_hb else ""
    labs = list(deck.type_of)
    for ia, a in enumerate(labs):
        for b in labs[ia:]:
            deck.coeffs.append(f"pair_coeff {deck.type_of[a]} {deck.type_of[b]} {prefix}"
                               f"{_dreiding_pair_args(ff, P, tindex[a], tindex[b], to_kcal)}")
    if with_hb:
        donors = sorted({top.types[d] for d in range(n) if int(hyd[d, 0]) >= 0})
        hydrogens = sorted({top.types[int(h)] for h in hyd[hyd >= 0]})
        acceptors = sorted({top.types[a] for a in range(n) if bool(model.hbond_acceptor[a])})
        d0 = float(P["hbond_d0"]) * to_kcal
        r0 = float(P["hbond_r0"])
        for d in donors:
            for a in acceptors:
                i, j = sorted((deck.type_of[d], deck.type_of[a]))
                for h in hydrogens:
                    deck.coeffs.append(f"pair_coeff {i} {j} hbond/dreiding/lj {deck.type_of[h]} i {d0:.14g} "
                                       f"{r0:.14g} 4 {hb_tail}")
    deck.coeffs += [f"bond_coeff {t} " + " ".join(map(str, key)) for t, key in k["bond"].items()]
    hybrid = len(angle_styles) > 1
    for t, key in k["angle"].items():
        args = " ".join(map(str, key[1:] if key[0] == "cosine/squared" else key[1:2]))
        deck.coeffs.append(f"angle_coeff {t} {key[0] + ' ' if hybrid else ''}{args}")
    deck.coeffs += [f"dihedral_coeff {t} " + " ".join(map(str, key)) for t, key in k["dihedral"].items()]
    deck.coeffs += [f"improper_coeff {t} " + " ".join(map(str, key)) for t, key in k["improper"].items()]
    return deck


# ----------------------------------------------------------------------------- entry points
def _box(pos: np.ndarray, cell: Optional[np.ndarray], pad: float):
    """Wrapped positions, ``[[lo, hi]] x 3`` and the boundary keywords."""
    if cell is None:
        return pos, np.stack([pos.min(0) - pad, pos.max(0) + pad], 1), "m m m"
    h = np.asarray(cell, float).reshape(3, 3)
    if np.count_nonzero(np.abs(h - np.diag(np.diag(h))) > 1e-12):
        raise ValueError("the LAMMPS inputs take an orthorhombic cell (a diagonal cell matrix)")
    lengths = np.diag(h).copy()
    return np.mod(pos, lengths), np.stack([np.zeros(3), lengths], 1), "p p p"


def _writer(model):
    from .amber import Amber
    from .charmm import Charmm
    from .dreiding import Dreiding
    from .opls import OPLS
    # Charmm derives from Amber: test the narrower class first
    for cls, fn in ((OPLS, _opls), (Charmm, _charmm), (Amber, _amber), (Dreiding, _dreiding)):
        if isinstance(model, cls):
            return fn
    raise TypeError(f"no LAMMPS input writer for {type(model).__name__} (OPLS, AMBER, CHARMM and DREIDING are written)")


def lammps_input(model, pos, cell=None):
    """``(data file text, commands, energy offset in kcal/mol)`` of a classical model at ``pos``
    (the commands name the data file ``DATAFILE`` in their ``read_data`` line)."""
    model = getattr(model, "model", model)
    as_np = lambda x: np.asarray(x.detach().cpu() if hasattr(x, "detach") else x, float)  # noqa: E731
    pos = as_np(pos).reshape(-1, 3)
    cell = None if cell is None else as_np(cell)
    if float(getattr(model, "switch_width", 0.0)) > 0.0:
        raise ValueError("a switched cutoff (switch_width > 0) has no LAMMPS style; use switch_width=0")
    fn = _writer(model)
    pos, bounds, boundary = _box(pos, cell, float(model.cutoff))
    deck = fn(model, boundary)
    return deck.data_text(pos, bounds), deck.commands(), deck.offset


def write_lammps_input(model, pos, cell=None, directory: Union[str, Path] = ".", name: str = "system") -> Path:
    """Writes ``name.data`` and ``in.name`` into ``directory``; returns the input script's path."""
    data, cmds, offset = lammps_input(model, pos, cell)
    out = Path(directory)
    out.mkdir(parents=True, exist_ok=True)
    (out / f"{name}.data").write_text(data)
    script = [c.replace("DATAFILE", f"{name}.data") for c in cmds]
    if offset:
        script = [f"# energy offset not in LAMMPS (the OPLS series constants V0): {offset:.15g} kcal/mol"] + script
    path = out / f"in.{name}"
    path.write_text("\n".join(script) + "\n")
    return path
