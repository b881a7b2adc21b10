"""LAMMPS data files and input commands for the fixed-topology force fields, so that a model (with
trained parameters) can be run or cross-checked in LAMMPS (``units real``, ``atom_style full``).

OPLS: ``pair_style lj/cut/coul/cut`` with geometric mixing, harmonic bonds and angles, ``dihedral_style
opls`` (the series constants ``V0``, which LAMMPS drops, are returned as an energy offset) and
``improper_style cvff``; AMBER: arithmetic mixing, ``dihedral_style fourier`` with each torsion's
terms and phases, ``improper_style cvff``; CHARMM: ``lj/charmm/coul/charmm`` with the pair table (NBFIX and own 1-4
values) written per type pair, Urey-Bradley terms in ``angle_style charmm``, ``dihedral_style
charmm`` carrying the 1-4 pairs (weight ``1/count`` for a pair closing several dihedrals), harmonic
impropers; DREIDING: ``lj/cut`` or ``buck`` (exp-6), Morse or harmonic bonds from the bond orders,
``cosine/squared`` angles (``cosine`` at linear centres), ``dihedral_style harmonic``,
``improper_style umbrella`` and ``hbond/dreiding/lj`` overlaid for hydrogen bonds. Charges are rescaled so that LAMMPS's Coulomb constant
(332.06371) reproduces the model's. Bonded types are deduplicated by their parameters. The file
layout and command set follow the reference (``src/xnn/ffnn/models/lammps_input.py``); cells must be
orthorhombic, a cluster gets a shrink-wrapped box.
"""
from __future__ import annotations

import math
from pathlib import Path
from typing import Optional, Union

import numpy as np

LAMMPS_COULOMB = 332.06371
_DEG = math.pi / 180.0
_SECTIONS = (("bond", "Bonds"), ("angle", "Angles"), ("dihedral", "Dihedrals"), ("improper", "Impropers"))


def _r(x, nd: int = 14) -> float:
    return round(float(x), nd)


def _box(pos: np.ndarray, cell: Optional[np.ndarray], pad: float):
    if cell is None:
        return pos, np.stack([pos.min(0) - pad, pos.max(0) + pad], 1), "m m m"
    cell = np.asarray(cell, float).reshape(3, 3)
    if np.abs(cell - np.diag(np.diag(cell))).max() > 1e-12:
        raise ValueError("the LAMMPS inputs take an orthorhombic cell (a diagonal cell matrix)")
    lengths = np.diag(cell)
    return pos % lengths, np.stack([np.zeros(3), lengths], 1), "p p p"


def _data(title: str, pos, bounds, masses: dict, types: list, charges, sections: dict, counts: dict) -> str:
    lines = [title, "", f"{len(types)} atoms"] + [f"{len(sections.get(s, []))} {s.lower()}" for _, s in _SECTIONS]
    lines += ["", f"{len(masses)} atom types"] + [f"{counts.get(s, 0)} {k} types" for k, s in _SECTIONS] + [""]
    lines += [f"{float(bounds[a, 0])!r} {float(bounds[a, 1])!r} {x}lo {x}hi" for a, x in enumerate("xyz")]
    lines += ["", "Masses", ""] + [f"{t} {m:.6f}" for t, m in masses.items()]
    lines += ["", "Atoms # full", ""]
    lines += [f"{i + 1} 1 {t} {q:.15g} {x:.14f} {y:.14f} {z:.14f}" for i, (t, q, (x, y, z)) in enumerate(zip(types, charges, pos))]
    for _, s in _SECTIONS:
        rows = sections.get(s, [])
        if rows:
            lines += ["", s, ""] + [" ".join(str(v) for v in (m + 1, *row)) for m, row in enumerate(rows)]
    return "\n".join(lines) + "\n"


def _styles(sections: dict, styles: dict) -> list:
    return [f"{k}_style {styles[k]}" for k, s in _SECTIONS if sections.get(s)]


def _opls(model, pos, bounds, boundary):
    from .opls import KCAL_TO_EV, KE
    ev = 1.0 / KCAL_TO_EV
    ff = model.ff
    P = {k: v.detach().double().cpu() for k, v in ff.params.items()}
    t_atom = model.top_type.tolist()
    used = list(dict.fromkeys(t_atom))
    at_id = {t: i + 1 for i, t in enumerate(used)}
    q = ff.charges.detach().double().cpu()[model.top_type.cpu()].numpy() * math.sqrt(KE * ev / LAMMPS_COULOMB)

    def rows(index, types, key):
        out, table = [], {}
        for m in range(index.shape[1]):
            k = key(int(types[m]))
            table.setdefault(k, len(table) + 1)
            out.append((table[k], *[int(a) + 1 for a in index[:, m]]))
        return out, table
    sec, tab = {}, {}
    sec["Bonds"], tab["bond"] = rows(model.bond_index, model.bond_type,
                                     lambda t: (_r(P["bond_k"][t] * ev), _r(P["bond_r0"][t])))
    sec["Angles"], tab["angle"] = rows(model.angle_index, model.angle_type,
                                       lambda t: (_r(P["angle_k"][t] * ev), _r(P["angle_theta0"][t] / _DEG)))
    sec["Dihedrals"], tab["dihedral"] = rows(model.dihedral_index, model.dihedral_type,
                                             lambda t: tuple(_r(P["dihedral_v"][t, s] * ev) for s in (1, 2, 3, 4)))
    sec["Impropers"], tab["improper"] = rows(model.improper_index, model.improper_type,
                                             lambda t: (_r(0.5 * P["improper_v2"][t] * ev),))
    v0 = float(P["dihedral_v"][model.dihedral_type.cpu(), 0].sum()) * ev
    data = _data("xnn OPLS", pos, bounds, {at_id[t]: float(ff.type_mass[t]) for t in used}, [at_id[t] for t in t_atom],
                 q, sec, {s: len(tab[k]) for k, s in _SECTIONS})
    cmds = ["units real", "atom_style full", f"boundary {boundary}", f"pair_style lj/cut/coul/cut {float(model.cutoff)!r}",
            "pair_modify mix geometric", f"special_bonds lj 0.0 0.0 {model.fudge_lj!r} coul 0.0 0.0 {model.fudge_qq!r}"]
    cmds += _styles(sec, {"bond": "harmonic", "angle": "harmonic", "dihedral": "opls", "improper": "cvff"})
    cmds.append("read_data DATAFILE")
    cmds += [f"pair_coeff {at_id[t]} {at_id[t]} {float(P['epsilon'][t]) * ev:.15g} {float(P['sigma'][t]):.15g}" for t in used]
    cmds += [f"bond_coeff {i} {k[0]:.15g} {k[1]:.15g}" for k, i in tab["bond"].items()]
    cmds += [f"angle_coeff {i} {k[0]:.15g} {k[1]:.15g}" for k, i in tab["angle"].items()]
    cmds += [f"dihedral_coeff {i} " + " ".join(f"{v:.15g}" for v in k) for k, i in tab["dihedral"].items()]
    cmds += [f"improper_coeff {i} {k[0]:.15g} -1 2" for k, i in tab["improper"].items()]
    return data, cmds, v0


def _amber(model, pos, bounds, boundary):
    from .amber import KCAL_TO_EV, KE_KCAL
    ev = 1.0 / KCAL_TO_EV
    ff, top = model.ff, model.topology
    P = {k: v.detach().double().cpu() for k, v in ff.params.items()}
    used = list(dict.fromkeys(top.types))
    at_id = {t: i + 1 for i, t in enumerate(used)}
    ti = {t: ff.type_index(t) for t in used}
    q = model.charges.detach().double().cpu().numpy() * math.sqrt(KE_KCAL / LAMMPS_COULOMB)
    sec = {s: [] for _, s in _SECTIONS}
    tb, ta, td, tm = {}, {}, {}, {}
    for m, (i, j) in enumerate(top.bonds):
        k = int(model.bond_type[m])
        key = (_r(P["bond_k"][k] * ev), _r(P["bond_r0"][k]))
        sec["Bonds"].append((tb.setdefault(key, len(tb) + 1), i + 1, j + 1))
    for m, (i, j, k) in enumerate(top.angles):
        t = int(model.angle_type[m])
        key = (_r(P["angle_k"][t] * ev), _r(P["angle_theta0"][t] / _DEG))
        sec["Angles"].append((ta.setdefault(key, len(ta) + 1), i + 1, j + 1, k + 1))
    for m, (i, j, k, l) in enumerate(top.dihedrals):
        t = int(model.dihedral_type[m])
        terms = tuple((_r(P["dihedral_k"][t, s] * ev), int(ff.dihedral_n[t, s]),
                       _r(math.degrees(math.atan2(float(ff.dihedral_sin[t, s]), float(ff.dihedral_cos[t, s])))))
                      for s in range(P["dihedral_k"].shape[1]) if float(P["dihedral_k"][t, s]) != 0.0)
        if terms:
            sec["Dihedrals"].append((td.setdefault(terms, len(td) + 1), i + 1, j + 1, k + 1, l + 1))
    for m, (i, j, k, l) in enumerate(model.impropers):
        t = int(model.improper_type[m])
        key = (_r(P["improper_k"][t, 0] * ev), int(round(float(ff.improper_cos[t, 0]))), int(ff.improper_n[t, 0]))
        sec["Impropers"].append((tm.setdefault(key, len(tm) + 1), i + 1, j + 1, k + 1, l + 1))
    counts = {"Bonds": len(tb), "Angles": len(ta), "Dihedrals": len(td), "Impropers": len(tm)}
    data = _data("xnn AMBER", pos, bounds, {at_id[t]: float(ff.type_mass[ti[t]]) for t in used},
                 [at_id[t] for t in top.types], q, sec, counts)
    cmds = ["units real", "atom_style full", f"boundary {boundary}", f"pair_style lj/cut/coul/cut {float(model.cutoff)!r}",
            "pair_modify mix arithmetic", f"special_bonds lj 0.0 0.0 {model.fudge_lj!r} coul 0.0 0.0 {model.fudge_qq!r}"]
    cmds += _styles(sec, {"bond": "harmonic", "angle": "harmonic", "dihedral": "fourier", "improper": "cvff"})
    cmds.append("read_data DATAFILE")
    sig = 2.0 / 2.0 ** (1.0 / 6.0)
    cmds += [f"pair_coeff {at_id[t]} {at_id[t]} {float(P['epsilon'][ti[t]]) * ev:.15g} {float(P['rstar'][ti[t]]) * sig:.15g}"
             for t in used]
    cmds += [f"bond_coeff {i} {k[0]:.15g} {k[1]:.15g}" for k, i in tb.items()]
    cmds += [f"angle_coeff {i} {k[0]:.15g} {k[1]:.15g}" for k, i in ta.items()]
    cmds += [f"dihedral_coeff {i} {len(k)} " + " ".join(f"{a:.15g} {n} {d:.15g}" for a, n, d in k) for k, i in td.items()]
    cmds += [f"improper_coeff {i} {k[0]:.15g} {k[1]} {k[2]}" for k, i in tm.items()]
    return data, cmds, 0.0


def _charmm(model, pos, bounds, boundary):
    from .charmm import KCAL_TO_EV
    ev = 1.0 / KCAL_TO_EV
    ff, top = model.ff, model.topology
    P = {k: v.detach().double().cpu() for k, v in ff.params.items()}
    used = list(dict.fromkeys(top.types))
    at_id = {t: i + 1 for i, t in enumerate(used)}
    ti = {t: ff.type_index(t) for t in used}
    q = model.charges.detach().double().cpu().numpy() * math.sqrt(float(model.coulomb_constant) / LAMMPS_COULOMB)
    rmin, eps, rmin14, eps14 = (x.detach().double().cpu() for x in ff.pair_tables())
    sec = {s: [] for _, s in _SECTIONS}
    tb, ta, td, tm = {}, {}, {}, {}
    for m, (i, j) in enumerate(top.bonds):
        k = int(model.bond_type[m])
        sec["Bonds"].append((tb.setdefault((_r(P["bond_k"][k] * ev), _r(P["bond_r0"][k])), len(tb) + 1), i + 1, j + 1))
    ub = {(int(model.ub_index[0, m]), int(model.ub_index[1, m])):
          (_r(P["ub_k"][int(model.ub_type[m])] * ev), _r(P["ub_s0"][int(model.ub_type[m])]))
          for m in range(model.ub_index.shape[1])}
    for m, (i, j, k) in enumerate(top.angles):
        t = int(model.angle_type[m])
        key = (_r(P["angle_k"][t] * ev), _r(P["angle_theta0"][t] / _DEG)) + ub.get((i, k), (0.0, 0.0))
        sec["Angles"].append((ta.setdefault(key, len(ta) + 1), i + 1, j + 1, k + 1))
    # dihedral_style charmm also carries the 1-4 pairs: a pair shared by several dihedrals gets
    # weight 1/count on each, pairs that are not 1-4 (rings) weight 0
    p14 = set(map(tuple, top.pairs14))
    share: dict = {}
    for i, _, _, l in top.dihedrals:
        share[(min(i, l), max(i, l))] = share.get((min(i, l), max(i, l)), 0) + 1
    for m, (i, j, k, l) in enumerate(top.dihedrals):
        t, pair = int(model.dihedral_type[m]), (min(i, l), max(i, l))
        w14 = 1.0 / share[pair] if pair in p14 else 0.0
        for s in range(P["dihedral_k"].shape[1]):
            if float(ff.dihedral_mask[t, s]) == 0.0:
                continue
            phase = int(round(math.degrees(math.atan2(float(ff.dihedral_sin[t, s]), float(ff.dihedral_cos[t, s]))))) % 360
            key = (_r(P["dihedral_k"][t, s] * ev), int(ff.dihedral_n[t, s]), phase, w14 if s == 0 else 0.0)
            sec["Dihedrals"].append((td.setdefault(key, len(td) + 1), i + 1, j + 1, k + 1, l + 1))
    for m, (i, j, k, l) in enumerate(model.impropers):
        t = int(model.improper_type[m])
        key = (_r(P["improper_k"][t] * ev), _r(math.degrees(math.atan2(float(ff.improper_sin[t]), float(ff.improper_cos[t])))))
        sec["Impropers"].append((tm.setdefault(key, len(tm) + 1), i + 1, j + 1, k + 1, l + 1))
    counts = {"Bonds": len(tb), "Angles": len(ta), "Dihedrals": len(td), "Impropers": len(tm)}
    data = _data("xnn CHARMM", pos, bounds, {at_id[t]: float(ff.type_mass[ti[t]]) for t in used},
                 [at_id[t] for t in top.types], q, sec, counts)
    rc = float(model.cutoff)
    cmds = ["units real", "atom_style full", f"boundary {boundary}",
            f"pair_style lj/charmm/coul/charmm {rc - 1e-6!r} {rc!r}", "special_bonds charmm"]
    cmds += _styles(sec, {"bond": "harmonic", "angle": "charmm", "dihedral": "charmm", "improper": "harmonic"})
    cmds.append("read_data DATAFILE")
    root = 2.0 ** (1.0 / 6.0)
    for a in used:
        for b in used:
            if at_id[a] <= at_id[b]:
                x, y = ti[a], ti[b]
                cmds.append(f"pair_coeff {at_id[a]} {at_id[b]} {float(eps[x, y]) * ev:.15g} {float(rmin[x, y]) / root:.15g} "
                            f"{float(eps14[x, y]) * ev:.15g} {float(rmin14[x, y]) / root:.15g}")
    cmds += [f"bond_coeff {i} {k[0]:.15g} {k[1]:.15g}" for k, i in tb.items()]
    cmds += [f"angle_coeff {i} {k[0]:.15g} {k[1]:.15g} {k[2]:.15g} {k[3]:.15g}" for k, i in ta.items()]
    cmds += [f"dihedral_coeff {i} {k[0]:.15g} {k[1]} {k[2]} {k[3]:.15g}" for k, i in td.items()]
    cmds += [f"improper_coeff {i} {k[0]:.15g} {k[1]:.15g}" for k, i in tm.items()]
    return data, cmds, 0.0


def _dreiding_pair(ff, P, ia: int, ib: int, ev: float) -> str:
    if ff.form == "x6":
        # exp-6 as LAMMPS buck: A exp(-r / rho) - C / r^6, per-type A and C combined geometrically
        zeta = [max(float(P["x6_zeta"][x]), 6.0 + 1e-6) for x in (ia, ib)]
        r0 = [float(P["vdw_r0"][x]) for x in (ia, ib)]
        d0 = [float(P["vdw_d0"][x]) * ev for x in (ia, ib)]
        A = [d0[m] * 6.0 / (zeta[m] - 6.0) * math.exp(zeta[m]) for m in (0, 1)]
        C = [d0[m] * zeta[m] / (zeta[m] - 6.0) * r0[m] ** 6 for m in (0, 1)]
        rho = 1.0 / (0.5 * (zeta[0] / r0[0] + zeta[1] / r0[1]))
        return f"{math.sqrt(A[0] * A[1]):.14g} {rho:.14g} {math.sqrt(C[0] * C[1]):.14g}"
    d0 = math.sqrt(float(P["vdw_d0"][ia] * P["vdw_d0"][ib])) * ev
    ra, rb = float(P["vdw_r0"][ia]), float(P["vdw_r0"][ib])
    r0 = math.sqrt(ra * rb) if ff.combination == "geometric" else 0.5 * (ra + rb)
    return f"{d0:.14g} {r0 / 2.0 ** (1.0 / 6.0):.14g}"


def _dreiding(model, pos, bounds, boundary):
    from .dreiding import KCAL_TO_EV, KE
    ev = 1.0 / KCAL_TO_EV
    ff, top = model.ff, model.topology
    P = {k: v.detach().double().cpu() for k, v in ff.params.items()}
    n, cutoff = len(top.types), float(model.cutoff)
    used = list(dict.fromkeys(top.types))
    at_id = {t: i + 1 for i, t in enumerate(used)}
    ti = {t: ff.type_index(t) for t in used}
    orders = list(top.bond_orders) or [1.0] * len(top.bonds)
    sec = {s: [] for _, s in _SECTIONS}
    tb, ta, td, tm = {}, {}, {}, {}
    morse = model.bond_style == "morse"
    for (i, j), o in zip(top.bonds, orders):
        r0 = float(P["radius"][ti[top.types[i]]] + P["radius"][ti[top.types[j]]]) - ff.delta
        k_n = o * float(P["bond_k"])
        if morse:
            d_n = o * float(P["bond_d"])
            key = (_r(d_n * ev), _r(math.sqrt(k_n / (2.0 * d_n))), _r(r0))
        else:
            key = (_r(0.5 * k_n * ev), _r(r0))
        sec["Bonds"].append((tb.setdefault(key, len(tb) + 1), i + 1, j + 1))
    ka = float(P["angle_k"]) * ev
    for m, (i, j, k) in enumerate(top.angles):
        th0 = float(P["theta0"][ti[top.types[j]]])
        key = (("cosine", _r(ka), 0.0) if bool(model.angle_linear[m])
               else ("cosine/squared", _r(0.5 * ka / math.sin(th0) ** 2), _r(th0 / _DEG)))
        sec["Angles"].append((ta.setdefault(key, len(ta) + 1), i + 1, j + 1, k + 1))
    for m in range(model.dihedral_index.shape[1]):
        i, j, k, l = (int(x) for x in model.dihedral_index[:, m])
        rule = int(model.dihedral_rule[m])
        v = float(model.dihedral_weight[m]) * float(P["torsion_v"][rule]) * ev
        key = (_r(0.5 * v), -int(ff.rule_sign[rule]), int(ff.rule_n[rule]))
        sec["Dihedrals"].append((td.setdefault(key, len(td) + 1), i + 1, j + 1, k + 1, l + 1))
    for m in range(model.inversion_index.shape[1]):
        c, a, b, d = (int(x) for x in model.inversion_index[:, m])
        x = ti[top.types[c]]
        key = (_r(float(P["oop_k"][x]) * ev / 3.0), _r(float(P["oop_psi0"][x]) / _DEG))
        sec["Impropers"].append((tm.setdefault(key, len(tm) + 1), c + 1, a + 1, b + 1, d + 1))
    q = (model.charge.detach().double().cpu().numpy() * math.sqrt(KE * ev / LAMMPS_COULOMB) if model.has_coulomb
         else np.zeros(n))
    counts = {"Bonds": len(tb), "Angles": len(ta), "Dihedrals": len(td), "Impropers": len(tm)}
    data = _data("xnn DREIDING", pos, bounds, {at_id[t]: float(ff.type_mass[ti[t]]) or 1.0 for t in used},
                 [at_id[t] for t in top.types], q, sec, counts)
    hyd = model.hbond_hydrogens.cpu()
    hb = model.use_hbond and bool((hyd >= 0).any())
    base = f"{'buck' if ff.form == 'x6' else 'lj/cut'}{'/coul/cut' if model.has_coulomb else ''} {cutoff!r}"
    hb_ang = math.acos(model.hbond_cos) / _DEG
    cmds = ["units real", "atom_style full", f"boundary {boundary}", "special_bonds lj/coul 0.0 0.0 1.0",
            (f"pair_style hybrid/overlay {base} hbond/dreiding/lj 4 {model.hbond_cutoff!r} {model.hbond_cutoff!r} "
             f"{hb_ang!r}") if hb else f"pair_style {base}"]
    if tb:
        cmds.append(f"bond_style {'morse' if morse else 'harmonic'}")
    styles = sorted({k[0] for k in ta})
    if ta:
        cmds.append(f"angle_style hybrid {' '.join(styles)}" if len(styles) > 1 else f"angle_style {styles[0]}")
    if td:
        cmds.append("dihedral_style harmonic")
    if tm:
        cmds.append("improper_style umbrella")
    cmds.append("read_data DATAFILE")
    sub = f"{base.split()[0]} " if hb else ""
    for a in used:
        for b in used:
            if at_id[a] <= at_id[b]:
                cmds.append(f"pair_coeff {at_id[a]} {at_id[b]} {sub}{_dreiding_pair(ff, P, ti[a], ti[b], ev)}")
    if hb:
        donors = {top.types[d] for d in range(n) if int(hyd[d, 0]) >= 0}
        hydrogens = {top.types[int(h)] for h in hyd[hyd >= 0]}
        acceptors = {top.types[a] for a in range(n) if bool(model.hbond_acceptor[a])}
        for d in sorted(donors):
            for a in sorted(acceptors):
                for h in sorted(hydrogens):
                    cmds.append(f"pair_coeff {min(at_id[d], at_id[a])} {max(at_id[d], at_id[a])} hbond/dreiding/lj "
                                f"{at_id[h]} i {float(P['hbond_d0']) * ev:.14g} {float(P['hbond_r0']):.14g} 4 "
                                f"{model.hbond_cutoff!r} {model.hbond_cutoff!r} {hb_ang!r}")
    cmds += [f"bond_coeff {t} " + " ".join(str(v) for v in k) for k, t in tb.items()]
    multi = len(styles) > 1
    for k, t in ta.items():
        args = f"{k[1]} {k[2]}" if k[0] == "cosine/squared" else f"{k[1]}"
        cmds.append(f"angle_coeff {t} {k[0] + ' ' if multi else ''}{args}")
    cmds += [f"dihedral_coeff {t} {k[0]} {k[1]} {k[2]}" for k, t in td.items()]
    cmds += [f"improper_coeff {t} {k[0]} {k[1]}" for k, t in tm.items()]
    return data, cmds, 0.0


def lammps_input(model, pos, cell=None):
    """``(data file text, commands, energy offset in kcal/mol)`` of an OPLS or AMBER model at ``pos``
    (``read_data DATAFILE`` names the data file in the commands)."""
    from .amber import Amber
    from .charmm import Charmm
    from .dreiding import Dreiding
    from .opls import OPLS
    model = getattr(model, "model", model)
    pos = np.asarray(pos.detach().cpu() if hasattr(pos, "detach") else pos, float).reshape(-1, 3)
    cell = None if cell is None else np.asarray(cell.detach().cpu() if hasattr(cell, "detach") else cell, float)
    if float(getattr(model, "switch_width", 0.0)) > 0.0:
        raise ValueError("a switched cutoff (switch_width > 0) has no LAMMPS style; use switch_width=0")
    pos, bounds, boundary = _box(pos, cell, float(model.cutoff))
    if isinstance(model, OPLS):
        return _opls(model, pos, bounds, boundary)
    if isinstance(model, Charmm):
        return _charmm(model, pos, bounds, boundary)
    if isinstance(model, Amber):
        return _amber(model, pos, bounds, boundary)
    if isinstance(model, Dreiding):
        return _dreiding(model, pos, bounds, boundary)
    raise TypeError(f"no LAMMPS input writer for {type(model).__name__} (OPLS, AMBER, CHARMM and DREIDING are written)")


def write_lammps_input(model, pos, cell=None, directory: Union[str, Path] = ".", name: str = "system") -> Path:
    """Writes ``name.data`` and ``in.name`` into ``directory``; returns the input script's path."""
    data, cmds, offset = lammps_input(model, pos, cell)
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    (directory / f"{name}.data").write_text(data)
    lines = [c.replace("DATAFILE", f"{name}.data") for c in cmds]
    if offset:
        lines.insert(0, f"# energy offset not in LAMMPS (the OPLS series constants V0): {offset:.15g} kcal/mol")
    script = directory / f"in.{name}"
    script.write_text("\n".join(lines) + "\n")
    return script
