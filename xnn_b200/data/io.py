"""Structure files: extended XYZ, RuNNer ``input.data``, and torch / numpy containers.

Every reader returns structure dicts for :func:`~xnn_b200.data.dataset.structure_to_graph`
(``pos`` Angstrom, ``atomic_numbers``, optional ``cell`` rows / ``pbc`` and labels ``energy``
eV, ``forces`` eV/A, ``stress`` eV/A^3, ``charges`` e, ``total_charge``).

* extended XYZ (the ASE convention, parsed here without ASE): the comment line carries
  ``key=value`` pairs (``Lattice="..."``, ``Properties=species:S:1:pos:R:3:forces:R:3``,
  ``energy=...``, ``stress="..."`` as 9 or Voigt 6 numbers, ``pbc="T T T"``), the atom lines the
  listed columns;
* RuNNer ``input.data`` (atomic units in the file, converted to Angstrom / eV unless
  ``units="atomic"``), with the column layouts of the reference's
  ``src/xnn/common/data/runner_io.py`` (a bare ``begin`` means ``x y z element charge energy
  fx fy fz``; ``begin position(3) element charge forces(3) ...`` names the columns);
* ``.pt`` (a list of structure dicts) and ``.npz`` (arrays ``pos``, ``atomic_numbers`` and
  labels stacked over structures of equal size).
"""
from __future__ import annotations

import re
import shlex
from pathlib import Path
from typing import Any, Dict, Iterable, List, Union

import numpy as np
import torch

from .elements import ATOMIC_NUMBERS, SYMBOLS

BOHR_A = 0.529177210903
HARTREE_EV = 27.211386245988


# ------------------------------------------------------------------------------- extxyz
def _parse_info(line: str) -> Dict[str, str]:
    out: Dict[str, str] = {}
    for tok in shlex.split(line):
        if "=" in tok:
            k, _, v = tok.partition("=")
            out[k.strip()] = v.strip()
        else:
            out[tok] = "T"
    return out


def _properties(spec: str):
    parts = spec.split(":")
    cols = []
    for i in range(0, len(parts), 3):
        cols.append((parts[i], parts[i + 1], int(parts[i + 2])))
    return cols


def read_extxyz(path: Union[str, Path], energy_key: str = "energy", forces_key: str = "forces",
                stress_key: str = "stress") -> List[Dict[str, Any]]:
    lines = Path(path).read_text().splitlines()
    out, i = [], 0
    while i < len(lines):
        if not lines[i].strip():
            i += 1
            continue
        n = int(lines[i].split()[0])
        info = _parse_info(lines[i + 1])
        cols = _properties(info.get("Properties", "species:S:1:pos:R:3"))
        rows = [lines[i + 2 + a].split() for a in range(n)]
        i += 2 + n
        data: Dict[str, Any] = {}
        c = 0
        for name, kind, width in cols:
            vals = [r[c:c + width] for r in rows]
            c += width
            if kind == "S":
                data[name] = [v[0] for v in vals]
            elif kind == "I":
                data[name] = np.array(vals, dtype=np.int64).reshape(n, width)
            elif kind == "L":
                data[name] = np.array([[x in ("T", "True", "1") for x in v] for v in vals]).reshape(n, width)
            else:
                data[name] = np.array(vals, dtype=np.float64).reshape(n, width)
        s: Dict[str, Any] = {"pos": torch.tensor(data["pos"], dtype=torch.float64)}
        if "Z" in data:
            s["atomic_numbers"] = torch.tensor(data["Z"][:, 0])
        else:
            s["atomic_numbers"] = torch.tensor([ATOMIC_NUMBERS[x] for x in data["species"]])
        if "Lattice" in info:
            s["cell"] = torch.tensor([float(x) for x in info["Lattice"].split()], dtype=torch.float64).reshape(3, 3)
            pbc = info.get("pbc", "T T T").split()
            s["pbc"] = torch.tensor([x in ("T", "True", "1") for x in pbc])
        if energy_key in info:
            s["energy"] = float(info[energy_key])
        if forces_key in data:
            s["forces"] = torch.tensor(data[forces_key], dtype=torch.float64)
        if stress_key in info:
            v = [float(x) for x in info[stress_key].split()]
            if len(v) == 6:          # Voigt xx yy zz yz xz xy
                xx, yy, zz, yz, xz, xy = v
                v = [xx, xy, xz, xy, yy, yz, xz, yz, zz]
            s["stress"] = torch.tensor(v, dtype=torch.float64).reshape(3, 3)
        for key in ("total_charge", "charge"):
            if key in info:
                s["total_charge"] = float(info[key])
                break
        if "charges" in data:
            s["charges"] = torch.tensor(data["charges"][:, 0], dtype=torch.float64)
        out.append(s)
    return out


def write_extxyz(structures: Iterable[Dict[str, Any]], path: Union[str, Path]) -> Path:
    chunks = []
    for s in structures:
        pos = np.asarray(torch.as_tensor(s["pos"]).double())
        z = np.asarray(torch.as_tensor(s["atomic_numbers"]))
        props = "species:S:1:pos:R:3"
        f = s.get("forces")
        if f is not None:
            props += ":forces:R:3"
            f = np.asarray(torch.as_tensor(f).double())
        info = [f"Properties={props}"]
        if s.get("cell") is not None:
            cell = np.asarray(torch.as_tensor(s["cell"]).double()).reshape(-1)
            info.append('Lattice="' + " ".join(f"{x:.12g}" for x in cell) + '"')
            pbc = s.get("pbc", [True, True, True])
            info.append('pbc="' + " ".join("T" if bool(b) else "F" for b in np.asarray(pbc).reshape(-1)) + '"')
        if s.get("energy") is not None:
            info.append(f"energy={float(s['energy']):.12g}")
        if s.get("stress") is not None:
            st = np.asarray(torch.as_tensor(s["stress"]).double()).reshape(-1)
            info.append('stress="' + " ".join(f"{x:.12g}" for x in st) + '"')
        lines = [str(len(z)), " ".join(info)]
        for a in range(len(z)):
            row = f"{SYMBOLS[int(z[a])]} " + " ".join(f"{x:.12g}" for x in pos[a])
            if f is not None:
                row += " " + " ".join(f"{x:.12g}" for x in f[a])
            lines.append(row)
        chunks.append("\n".join(lines))
    p = Path(path)
    p.write_text("\n".join(chunks) + "\n")
    return p


# ------------------------------------------------------------------------------- RuNNer
_RUNNER_DEFAULT = (("position", 3), ("element", 1), ("charge", 1), ("energy", 1), ("forces", 3))
_RUNNER_ALIASES = {"positions": "position", "pos": "position", "charges": "charge", "force": "forces",
                   "elements": "element", "atomic_energy": "energy", "energies": "energy"}


def _runner_columns(tokens: List[str]):
    if not tokens:
        return _RUNNER_DEFAULT
    cols = []
    for t in tokens:
        m = re.fullmatch(r"([A-Za-z_]+)(?:\((\d+)\))?", t)
        if m is None:
            raise ValueError(f"unreadable RuNNer column {t!r}")
        name = _RUNNER_ALIASES.get(m.group(1).lower(), m.group(1).lower())
        cols.append((name, int(m.group(2) or 1)))
    return tuple(cols)


def read_runner(path: Union[str, Path], units: str = "xnn", charges: bool = True) -> List[Dict[str, Any]]:
    if units not in ("xnn", "atomic"):
        raise ValueError("units must be 'xnn' or 'atomic'")
    L = BOHR_A if units == "xnn" else 1.0
    E = HARTREE_EV if units == "xnn" else 1.0
    out: List[Dict[str, Any]] = []
    cur = None
    for raw in Path(path).read_text().splitlines():
        tok = raw.split()
        if not tok:
            continue
        key = tok[0].lower()
        if key == "begin":
            cur = {"cols": _runner_columns(tok[1:]), "lattice": [], "atoms": [], "energy": None, "charge": None,
                   "comment": None}
        elif cur is None:
            continue
        elif key == "comment":
            cur["comment"] = raw.split(None, 1)[1] if len(tok) > 1 else ""
        elif key == "lattice":
            cur["lattice"].append([float(x) for x in tok[1:4]])
        elif key == "atom":
            cur["atoms"].append(tok[1:])
        elif key == "energy":
            cur["energy"] = float(tok[1])
        elif key == "charge":
            cur["charge"] = float(tok[1])
        elif key == "end":
            pos, z, q, f = [], [], [], []
            for a in cur["atoms"]:
                c = 0
                for name, width in cur["cols"]:
                    vals = a[c:c + width]
                    c += width
                    if name == "position":
                        pos.append([float(x) for x in vals])
                    elif name == "element":
                        z.append(ATOMIC_NUMBERS[vals[0]])
                    elif name == "charge":
                        q.append(float(vals[0]))
                    elif name == "forces":
                        f.append([float(x) for x in vals])
            s: Dict[str, Any] = {"pos": torch.tensor(pos, dtype=torch.float64) * L, "atomic_numbers": torch.tensor(z)}
            if len(cur["lattice"]) == 3:
                s["cell"] = torch.tensor(cur["lattice"], dtype=torch.float64) * L
                s["pbc"] = torch.ones(3, dtype=torch.bool)
            if cur["energy"] is not None:
                s["energy"] = cur["energy"] * E
            if f:
                s["forces"] = torch.tensor(f, dtype=torch.float64) * (E / L)
            if q and charges:
                s["charges"] = torch.tensor(q, dtype=torch.float64)
            if cur["charge"] is not None:
                s["total_charge"] = cur["charge"]
            if cur["comment"] is not None:
                s["comment"] = cur["comment"]
            out.append(s)
            cur = None
    return out


def write_runner(structures: Iterable[Dict[str, Any]], path: Union[str, Path], units: str = "xnn") -> Path:
    L = BOHR_A if units == "xnn" else 1.0
    E = HARTREE_EV if units == "xnn" else 1.0
    lines = []
    for s in structures:
        lines.append("begin")
        if s.get("comment"):
            lines.append(f"comment {s['comment']}")
        if s.get("cell") is not None:
            for row in np.asarray(torch.as_tensor(s["cell"]).double()) / L:
                lines.append("lattice " + " ".join(f"{x:.15g}" for x in row))
        pos = np.asarray(torch.as_tensor(s["pos"]).double()) / L
        z = np.asarray(torch.as_tensor(s["atomic_numbers"]))
        f = s.get("forces")
        f = np.asarray(torch.as_tensor(f).double()) / (E / L) if f is not None else np.zeros_like(pos)
        q = s.get("charges")
        q = np.asarray(torch.as_tensor(q).double()) if q is not None else np.zeros(len(z))
        for a in range(len(z)):
            lines.append("atom " + " ".join(f"{x:.15g}" for x in pos[a]) + f" {SYMBOLS[int(z[a])]} {q[a]:.15g} "
                         f"0.0 " + " ".join(f"{x:.15g}" for x in f[a]))
        lines.append(f"energy {float(s.get("energy", 0.0)) / E:.15g}")
        lines.append(f"charge {float(s.get('total_charge', 0.0)):.10f}")
        lines.append("end")
    p = Path(path)
    p.write_text("\n".join(lines) + "\n")
    return p


# ------------------------------------------------------------------------------- dispatch
def read_structures(path: Union[str, Path], energy_key: str = "energy", forces_key: str = "forces",
                    stress_key: str = "stress") -> List[Dict[str, Any]]:
    p = Path(path)
    name = p.name.lower()
    if name.endswith((".xyz", ".extxyz")):
        return read_extxyz(p, energy_key, forces_key, stress_key)
    if name == "input.data" or name.endswith(".data"):
        return read_runner(p)
    if name.endswith(".pt"):
        return list(torch.load(p, weights_only=False))
    if name.endswith(".npz"):
        d = np.load(p)
        n = d["pos"].shape[0]
        out = []
        for i in range(n):
            s = {"pos": torch.tensor(d["pos"][i], dtype=torch.float64),
                 "atomic_numbers": torch.tensor(d["atomic_numbers"][i] if d["atomic_numbers"].ndim == 2
                                                else d["atomic_numbers"])}
            for k in ("energy", "forces", "stress", "cell"):
                if k in d.files:
                    s[k] = torch.tensor(d[k][i]) if k != "energy" else float(d[k][i])
            out.append(s)
        return out
    raise ValueError(f"unknown structure file type: {p}")
