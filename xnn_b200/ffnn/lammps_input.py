"""LAMMPS data files and input commands for the fixed-topology force fields, so that a model (with
trained parameters) can be run or cross-checked in LAMMPS (``units real``, ``atom_style full``).

OPLS: ``pair_style lj/cut/coul/cut`` with geometric mixing, harmonic bonds and angles, ``dihedral_style
opls`` (the series constants ``V0``, which LAMMPS drops, are returned as an energy offset) and
``improper_style cvff``; AMBER: arithmetic mixing, ``dihedral_style fourier`` with each torsion's
terms and phases, ``improper_style cvff``. Charges are rescaled so that LAMMPS's Coulomb constant
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


def lammps_input(model, pos, cell=None):
    """``(data file text, commands, energy offset in kcal/mol)`` of an OPLS or AMBER model at ``pos``
    (``read_data DATAFILE`` names the data file in the commands)."""
    from .amber import Amber
    from .charmm import Charmm
    from .opls import OPLS
    model = getattr(model, "model", model)
    pos = np.asarray(pos.detach().cpu() if hasattr(pos, "detach") else pos, float).reshape(-1, 3)
    cell = None if cell is None else np.asarray(cell.detach().cpu() if hasattr(cell, "detach") else cell, float)
    if float(getattr(model, "switch_width", 0.0)) > 0.0:
        raise ValueError("a switched cutoff (switch_width > 0) has no LAMMPS style; use switch_width=0")
    pos, bounds, boundary = _box(pos, cell, float(model.cutoff))
    if isinstance(model, OPLS):
        return _opls(model, pos, bounds, boundary)
    if isinstance(model, Amber) and not isinstance(model, Charmm):
        return _amber(model, pos, bounds, boundary)
    raise TypeError(f"no LAMMPS input writer for {type(model).__name__} (OPLS and AMBER are written)")


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
