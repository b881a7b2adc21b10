"""Reader of MolSSI/SEAMM ``.frc`` force-field files (format version 1).

A file opens with ``!MolSSI forcefield 1``; every section starts at a ``#`` line and runs to the next:
``#define <name>`` lists, per functional form, which labelled sections make up a variant (a row
``version ref form label [label:optional ...]``, newest version per form); ``#<form> <label>``
holds data rows ``version ref key... values...`` (newest version per key), ``!`` comments whose
last non-rule line names the columns, ``>`` annotations and ``@`` modifiers (``@units``,
``@type``, ``@combination``); ``#templates`` / ``#fragments`` carry JSON; ``#include`` pulls in
another file; ``#reference`` blocks cite sources. Keys are ordered canonically per symmetry
(bond, angle, torsion, improper with the centre third, out-of-plane with the centre second) so a
row written in either orientation resolves to one entry; ``*`` is the wildcard.

The grammar, the section kinds with their column names and default units, the canonical key
orders and the wildcard precedences of the lookups are those of the format (as read by the
reference's ``src/xnn/ffnn/common/frc.py:90-1770``); values are normalised on reading to Å,
kcal/mol, degrees, e and Da, nonbond rows to (sigma, epsilon).
"""
from __future__ import annotations

import json
import math
import re
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Sequence, Tuple, Union

WILDCARD = "*"
FORMAT_VERSION = 1
DATA_DIR = Path(__file__).resolve().parent / "data"

# ----------------------------------------------------------------------------------------- units
# (scale to kcal/mol, Å, degree, e, Da; dimension exponents of those five)
_UNITS = {
    "kcal/mol": (1.0, (1, 0, 0, 0, 0)), "kJ/mol": (1.0 / 4.184, (1, 0, 0, 0, 0)),
    "eV": (23.060547830619026, (1, 0, 0, 0, 0)), "hartree": (627.5094740631, (1, 0, 0, 0, 0)),
    "Å": (1.0, (0, 1, 0, 0, 0)), "angstrom": (1.0, (0, 1, 0, 0, 0)), "A": (1.0, (0, 1, 0, 0, 0)),
    "nm": (10.0, (0, 1, 0, 0, 0)), "pm": (0.01, (0, 1, 0, 0, 0)), "bohr": (0.529177210903, (0, 1, 0, 0, 0)),
    "degree": (1.0, (0, 0, 1, 0, 0)), "degrees": (1.0, (0, 0, 1, 0, 0)), "deg": (1.0, (0, 0, 1, 0, 0)),
    "radian": (180.0 / math.pi, (0, 0, 1, 0, 0)), "rad": (180.0 / math.pi, (0, 0, 1, 0, 0)),
    "e": (1.0, (0, 0, 0, 1, 0)), "Da": (1.0, (0, 0, 0, 0, 1)), "Dalton": (1.0, (0, 0, 0, 0, 1)),
    "amu": (1.0, (0, 0, 0, 0, 1)), "g/mol": (1.0, (0, 0, 0, 0, 1)),
}
_UNIT_NAME = re.compile(r"kcal/mol|kJ/mol|g/mol|[A-Za-zÅ]+")


def parse_unit(text: str) -> Tuple[float, Tuple[float, ...]]:
    """``(scale, dimension)`` of a unit expression: products, quotients, parentheses and powers
    ``^n``, ``**n``, ``**(p/q)`` of the base units (``kJ/mol/nm^2``, ``(kcal/mol)**(1/12)*Å``)."""
    s = text.strip().replace("**", "^")
    i = [0]

    def ws():
        while i[0] < len(s) and s[i[0]] == " ":
            i[0] += 1

    def num():
        ws()
        m = re.match(r"[+-]?\d+(\.\d+)?", s[i[0]:])
        if not m:
            raise ValueError(f"bad exponent in unit {text!r}")
        i[0] += m.end()
        return float(m.group(0))

    def power():
        ws()
        if s[i[0]:i[0] + 1] == "(":
            i[0] += 1
            p, q = num(), 1.0
            ws()
            if s[i[0]:i[0] + 1] == "/":
                i[0] += 1
                q = num()
            ws()
            if s[i[0]:i[0] + 1] != ")":
                raise ValueError(f"unbalanced exponent in unit {text!r}")
            i[0] += 1
            return p / q
        return num()

    def factor():
        ws()
        if s[i[0]:i[0] + 1] == "(":
            i[0] += 1
            val = product()
            ws()
            if s[i[0]:i[0] + 1] != ")":
                raise ValueError(f"unbalanced parentheses in unit {text!r}")
            i[0] += 1
        else:
            m = _UNIT_NAME.match(s, i[0])
            if not m or m.group(0) not in _UNITS:
                raise ValueError(f"cannot read unit {text!r} at {s[i[0]:]!r}")
            i[0] = m.end()
            sc, dim = _UNITS[m.group(0)]
            val = (sc, tuple(float(d) for d in dim))
        ws()
        if s[i[0]:i[0] + 1] == "^":
            i[0] += 1
            e = power()
            val = (val[0] ** e, tuple(d * e for d in val[1]))
        return val

    def product():
        sc, dim = factor()
        while True:
            ws()
            op = s[i[0]:i[0] + 1]
            if op not in ("*", "/"):
                return sc, dim
            i[0] += 1
            s2, d2 = factor()
            sign = 1.0 if op == "*" else -1.0
            sc = sc * s2 if op == "*" else sc / s2
            dim = tuple(a + sign * b for a, b in zip(dim, d2))

    if not s:
        return 1.0, (0.0,) * 5
    out = product()
    ws()
    if i[0] != len(s):
        raise ValueError(f"trailing text in unit {text!r}")
    return out


def convert_units(value: float, src: str, dst: str) -> float:
    s1, d1 = parse_unit(src)
    s2, d2 = parse_unit(dst)
    if any(abs(a - b) > 1e-12 for a, b in zip(d1, d2)):
        raise ValueError(f"cannot convert {src!r} to {dst!r}: different dimensions")
    return value * s1 / s2


def nonbond_to_sigma_eps(form: str, v1: float, v2: float, u1: Optional[str] = None,
                         u2: Optional[str] = None) -> Tuple[float, float]:
    """A nonbond row of ``@type form`` as ``(sigma [Å], epsilon [kcal/mol])``."""
    if form == "sigma-eps":
        return convert_units(v1, u1 or "Å", "Å"), convert_units(v2, u2 or "kcal/mol", "kcal/mol")
    if form in ("rmin-eps", "eps-rmin"):
        if form == "eps-rmin":
            v1, v2, u1, u2 = v2, v1, u2, u1
        return (convert_units(v1, u1 or "Å", "Å") / 2.0 ** (1.0 / 6.0),
                convert_units(v2, u2 or "kcal/mol", "kcal/mol"))
    if form in ("A-B", "A/r-B/r"):
        if form == "A/r-B/r":
            a = convert_units(v1, u1 or "(kcal/mol)**(1/12)*Å", "(kcal/mol)**(1/12)*Å") ** 12
            b = convert_units(v2, u2 or "(kcal/mol)**(1/6)*Å", "(kcal/mol)**(1/6)*Å") ** 6
        else:
            a = convert_units(v1, u1 or "kcal/mol*Å^12", "kcal/mol*Å^12")
            b = convert_units(v2, u2 or "kcal/mol*Å^6", "kcal/mol*Å^6")
        if a == 0.0 or b == 0.0:
            return 0.0, 0.0
        return (a / b) ** (1.0 / 6.0), b * b / (4.0 * a)
    raise ValueError(f"unknown nonbond form {form!r}")


def parse_version(text: str) -> tuple:
    """A comparable key of a version token (``2023.01.29``, ``1.0``)."""
    return tuple(int(x) if x.isdigit() else 0 for x in re.split(r"[.\-]", str(text)))


# --------------------------------------------------------------------------------------- schema
def _c(*cols):
    return [(c[0], c[1], c[2] if len(c) > 2 else float) for c in cols]


# kind -> key width, key symmetry, interaction class, value columns (name, default unit, type) or
# None (names from the header), trailing text column, value swap on a flipped key
SCHEMA: Dict[str, dict] = {
    "atom_types": dict(n=1, sym="none", cls="atom type", cols=_c(("Mass", "Da"), ("El", "", str),
                                                                 ("connections", "", str)), text="Comment"),
    "equivalence": dict(n=1, sym="none", cls="equivalence",
                        cols=_c(*[(x, "", str) for x in ("NonB", "Bond", "Angle", "Torsion", "OOP")])),
    "auto_equivalence": dict(n=1, sym="none", cls="auto equivalence", cols=None),
    "metadata": dict(n=1, sym="none", cls="metadata", cols=[("Value", "", None)], text="Description"),
    "charges": dict(n=1, sym="none", cls="atomic charge", cols=_c(("Q", "e"))),
    "bond_increments": dict(n=2, sym="like_bond", cls="bond charge increment",
                            cols=_c(("deltaij", "e"), ("deltaji", "e")), flip=1),
    "nonbond(12-6)": dict(n=1, sym="none", cls="pair", form="sigma-eps", cols=_c(("sigma", "Å"), ("eps", "kcal/mol"))),
    "nonbond_1-4(12-6)": dict(n=1, sym="none", cls="pair 1-4", form="sigma-eps",
                              cols=_c(("sigma", "Å"), ("eps", "kcal/mol"))),
    "nonbond_pair(12-6)": dict(n=2, sym="like_bond", cls="pair",
                               cols=_c(("rmin", "Å"), ("eps", "kcal/mol"), ("rmin14", "Å"), ("eps14", "kcal/mol"))),
    "nonbond(9-6)": dict(n=1, sym="none", cls="pair", form="rmin-eps", cols=_c(("rmin", "Å"), ("eps", "kcal/mol"))),
    "buckingham": dict(n=None, sym="like_bond", cls="pair", cols=None),
    "dreiding_atomic_parameters": dict(n=1, sym="none", cls="dreiding atomic",
                                       cols=_c(("Radius", "Å"), ("Theta0", "degree"))),
    "dreiding_out_of_plane": dict(n=4, sym="like_oop", cls="out-of-plane",
                                  cols=_c(("K2", "kcal/mol/radian^2"), ("Psi0", "degree"))),
    "quadratic_bond": dict(n=2, sym="like_bond", cls="bond", cols=_c(("R0", "Å"), ("K2", "kcal/mol/Å^2"))),
    "quartic_bond": dict(n=2, sym="like_bond", cls="bond", cols=_c(("R0", "Å"), ("K2", "kcal/mol/Å^2"),
                                                                   ("K3", "kcal/mol/Å^3"), ("K4", "kcal/mol/Å^4"))),
    "quadratic_angle": dict(n=3, sym="like_angle", cls="angle",
                            cols=_c(("Theta0", "degree"), ("K2", "kcal/mol/radian^2"))),
    "urey_bradley": dict(n=3, sym="like_angle", cls="urey-bradley", cols=_c(("S0", "Å"), ("K2", "kcal/mol/Å^2"))),
    "quartic_angle": dict(n=3, sym="like_angle", cls="angle",
                          cols=_c(("Theta0", "degree"), ("K2", "kcal/mol/radian^2"), ("K3", "kcal/mol/radian^3"),
                                  ("K4", "kcal/mol/radian^4"))),
    "simple_fourier_angle": dict(n=3, sym="like_angle", cls="angle", cols=_c(("K", "kcal/mol"), ("n", "", int))),
    "tabulated_angle": dict(n=3, sym="like_angle", cls="angle",
                            cols=_c(("Eqn", "", str), ("K", "kcal/mol"), ("n", "", int), ("Rb", "Å"),
                                    ("A", "kcal/mol*Å^12"), ("zero-shift", "degree"))),
    "torsion_opls": dict(n=4, sym="like_torsion", cls="torsion",
                         cols=_c(("V1", "kcal/mol"), ("V2", "kcal/mol"), ("V3", "kcal/mol"), ("V4", "kcal/mol"))),
    "torsion_1": dict(n=4, sym="like_torsion", cls="torsion",
                      cols=_c(("KPhi", "kcal/mol"), ("n", "", int), ("Phi0", "degree"))),
    "torsion_3": dict(n=4, sym="like_torsion", cls="torsion",
                      cols=_c(("V1", "kcal/mol"), ("Phi0_1", "degree"), ("V2", "kcal/mol"), ("Phi0_2", "degree"),
                              ("V3", "kcal/mol"), ("Phi0_3", "degree"))),
    "improper_opls": dict(n=4, sym="like_improper", cls="out-of-plane", cols=_c(("V2", "kcal/mol"))),
    "torsion_fourier": dict(n=4, sym="like_torsion", cls="torsion",
                            cols=_c(*[c for m in range(1, 7) for c in ((f"K{m}", "kcal/mol"), (f"n{m}", "", int),
                                                                        (f"Phi0_{m}", "degree"))])),
    "improper_fourier": dict(n=4, sym="none", cls="out-of-plane",
                             cols=_c(("K1", "kcal/mol"), ("n1", "", int), ("Phi0_1", "degree"), ("K2", "kcal/mol"),
                                     ("n2", "", int), ("Phi0_2", "degree"))),
    "improper_harmonic": dict(n=4, sym="none", cls="out-of-plane",
                              cols=_c(("K2", "kcal/mol/radian^2"), ("Chi0", "degree"))),
    "wilson_out_of_plane": dict(n=4, sym="like_oop", cls="out-of-plane",
                                cols=_c(("K", "kcal/mol/radian^2"), ("Chi0", "degree"))),
    "amoeba_bond": dict(n=2, sym="like_bond", cls="bond", cols=_c(("R0", "Å"), ("K2", "kcal/mol/Å^2"))),
    "amoeba_angle": dict(n=3, sym="like_angle", cls="angle",
                         cols=_c(("K2", "kcal/mol/radian^2"), ("Theta0_1", "degree"), ("Theta0_2", "degree"),
                                 ("Theta0_3", "degree"))),
    "amoeba_angle_inplane": dict(n=3, sym="like_angle", cls="angle",
                                 cols=_c(("K2", "kcal/mol/radian^2"), ("Theta0_1", "degree"), ("Theta0_2", "degree"))),
    "stretch_bend": dict(n=3, sym="like_angle", cls="stretch-bend",
                         cols=_c(("K1", "kcal/mol/Å/radian"), ("K2", "kcal/mol/Å/radian")), flip=1),
    "amoeba_out_of_plane": dict(n=4, sym="none", cls="out-of-plane", cols=_c(("K2", "kcal/mol/radian^2"))),
    "pi_torsion": dict(n=2, sym="like_bond", cls="torsion", cols=_c(("K2", "kcal/mol"))),
    "buffered_14-7": dict(n=1, sym="none", cls="pair", cols=_c(("rmin", "Å"), ("eps", "kcal/mol"), ("reduction", ""))),
    "buffered_14-7_pair": dict(n=2, sym="like_bond", cls="pair", cols=_c(("rmin", "Å"), ("eps", "kcal/mol"))),
    "atomic_multipole": dict(n=4, sym="none", cls="multipole",
                             cols=_c(("Q", "e"), ("Dx", "e*bohr"), ("Dy", "e*bohr"), ("Dz", "e*bohr"),
                                     ("Qxx", "e*bohr^2"), ("Qxy", "e*bohr^2"), ("Qxz", "e*bohr^2"),
                                     ("Qyy", "e*bohr^2"), ("Qyz", "e*bohr^2"), ("Qzz", "e*bohr^2"))),
    "polarizability": dict(n=1, sym="none", cls="polarize", cols=_c(("alpha", "Å^3"), ("thole", "")), text="Group"),
    "charge_penetration": dict(n=1, sym="none", cls="penetration", cols=_c(("Core", "e"), ("alpha", "1/Å"))),
    "charge_transfer": dict(n=1, sym="none", cls="transfer", cols=_c(("eps", "kcal/mol"), ("alpha", "1/Å"))),
    "pauli_repulsion": dict(n=1, sym="none", cls="repulsion",
                            cols=_c(("K", "kcal/mol*Å"), ("alpha", "1/Å"), ("valence", "e"))),
    "damped_dispersion": dict(n=1, sym="none", cls="dispersion", cols=_c(("C6", "(kcal/mol)^1/2*Å^3"), ("alpha", "1/Å"))),
    "bond_charge_flux": dict(n=2, sym="like_bond", cls="charge flux", cols=_c(("J", "e/Å")), sign_flip=True),
    "angle_charge_flux": dict(n=3, sym="like_angle", cls="charge flux",
                              cols=_c(("Jt1", "e/radian"), ("Jt2", "e/radian"), ("Jb1", "e/Å"), ("Jb2", "e/Å")),
                              flip=1, flip_pairs=2),
    "reaxff_general_parameters": dict(n=1, sym="none", cls="reaxff general", cols=_c(("Value", "")),
                                      text="Description"),
    "reaxff_off-diagonal_parameters": dict(n=2, sym="none", cls="reaxff off-diagonal", cols=None),
    "reaxff_angle_parameters": dict(n=3, sym="none", cls="reaxff angle", cols=None),
    "reaxff_torsion_parameters": dict(n=4, sym="none", cls="reaxff torsion", cols=None),
    "reaxff_hydrogen-bond_parameters": dict(n=3, sym="none", cls="reaxff hydrogen bond", cols=None),
}
for _g in ("1-8", "9-16", "17-24", "25-32"):
    SCHEMA[f"reaxff_atomic_parameters_{_g}"] = dict(n=1, sym="none", cls="reaxff atomic", cols=None)
for _g in ("1-8", "9-16"):
    SCHEMA[f"reaxff_bond_parameters_{_g}"] = dict(n=2, sym="none", cls="reaxff bond", cols=None)

JSON_SECTIONS = ("templates", "fragments", "torsion_torsion")
_FORM_PARAMS = {"sigma-eps": ("sigma", "eps"), "rmin-eps": ("rmin", "eps"), "eps-rmin": ("eps", "rmin"),
                "A-B": ("A", "B"), "A/r-B/r": ("A", "B")}
_KEY_TOKENS = {"I", "J", "K", "L", "M", "N", "Type", "Center", "Parameter", "Atom"}
_RULE = re.compile(r"^\s*-+[\s-]*$")


def _auto(tok: str):
    try:
        return int(tok)
    except ValueError:
        pass
    try:
        return float(tok)
    except ValueError:
        return tok


def canonical_key(sym: str, atoms: Sequence[str]) -> Tuple[tuple, bool]:
    """The canonical order of a key under its symmetry and whether it was flipped."""
    a = list(atoms)
    if len(a) == 2 and sym == "like_bond":
        return ((a[1], a[0]), True) if a[0] > a[1] else ((a[0], a[1]), False)
    if len(a) == 3 and sym == "like_angle":
        return ((a[2], a[1], a[0]), True) if a[0] > a[2] else (tuple(a), False)
    if len(a) == 4:
        i, j, k, l = a
        if sym == "like_torsion":
            if (j == k and i > l) or j > k:
                return (l, k, j, i), True
            return tuple(a), False
        if sym == "like_improper":            # centre third
            o = sorted((i, j, l))
            key = (o[0], o[1], k, o[2])
            return key, list(key) != a
        if sym == "like_oop":                 # centre second
            o = sorted((i, k, l))
            key = (o[0], j, o[1], o[2])
            return key, list(key) != a
    return tuple(a), False


def _flip_values(sch: dict, vals: list) -> list:
    vals = list(vals)
    f = int(sch.get("flip", 0) or 0)
    if f:
        for p in range(int(sch.get("flip_pairs", 1))):
            a = 2 * p * f
            if len(vals) >= a + 2 * f:
                vals[a:a + f], vals[a + f:a + 2 * f] = vals[a + f:a + 2 * f], vals[a:a + f]
    if sch.get("sign_flip"):
        vals = [(v[1:] if v.startswith("-") else "-" + v) for v in vals]
    return vals


# ----------------------------------------------------------------------------------------- data
@dataclass
class Row:
    version: str
    reference: str
    key: tuple
    values: dict
    source: str = ""

    @property
    def version_key(self) -> tuple:
        return parse_version(self.version)


@dataclass
class Section:
    kind: str
    label: str
    comments: list = field(default_factory=list)
    annotations: list = field(default_factory=list)
    modifiers: dict = field(default_factory=dict)
    key_columns: list = field(default_factory=list)
    columns: list = field(default_factory=list)
    rows: list = field(default_factory=list)
    data: object = None
    source: str = ""

    def modifier(self, word: str) -> Optional[list]:
        items = self.modifiers.get(word)
        return items[0] if items else None


@dataclass
class Reference:
    number: str
    text: str
    author: str = ""
    date: str = ""
    source: str = ""


class FrcFile:
    """A parsed ``.frc`` file and everything it includes."""

    def __init__(self, path: Union[str, Path], include_dirs: Sequence[Union[str, Path]] = ()):
        self.path = Path(path)
        self.include_dirs = [Path(p) for p in include_dirs]
        self.header, self.format_version = "", None
        self.sections: Dict[Tuple[str, str], Section] = {}
        self.defines: Dict[str, List[tuple]] = {}
        self.references: Dict[Tuple[str, str], Reference] = {}
        self.missing_includes: List[str] = []
        self.files: List[Path] = []
        self._read(self.path, top=True)

    @property
    def forcefields(self) -> List[str]:
        return list(self.defines)

    def _include(self, target: str, current: Path) -> Optional[Path]:
        name = target.split(":", 1)[1] if ":" in target else target
        for base in [current.parent] + self.include_dirs + [DATA_DIR]:
            p = base / name
            if p.is_file():
                return p
        return None

    def _read(self, path: Path, top: bool = False) -> None:
        if not path.is_file():
            raise FileNotFoundError(str(path))
        self.files.append(path)
        lines = path.read_text(encoding="utf-8").splitlines()
        if top and lines:
            self.header = lines[0].strip()
            m = re.match(r"!\s*(\S+)\s+forcefield\s*(\d+)?", self.header)
            self.format_version = int(m.group(2)) if m and m.group(2) else None
        i, n = (1 if top else 0), len(lines)
        while i < n and not lines[i].lstrip().startswith("#"):
            i += 1
        while i < n:
            words = lines[i].strip()[1:].split()
            j = i + 1
            while j < n and not lines[j].lstrip().startswith("#"):
                j += 1
            body, i = lines[i + 1:j], j
            kind = words[0] if words else ""
            if kind in ("", "end", "version"):
                continue
            if kind == "include":
                found = self._include(words[1] if len(words) > 1 else "", path)
                if found is None:
                    if "missing_ok" in words[2:]:
                        self.missing_includes.append(words[1])
                        continue
                    raise FileNotFoundError(f"{path}: cannot find included file {words[1]!r}")
                self._read(found)
                continue
            label = words[1] if len(words) > 1 else "missing"
            if kind == "define":
                if label in self.defines:
                    raise ValueError(f"{path}: force field {label!r} is defined twice")
                self.defines[label] = [tuple(w[:3]) + (w[3:],) for w in
                                       (ln.split() for ln in body if ln.strip() and ln.strip()[0] not in "!>@")
                                       if len(w) >= 4]
            elif kind == "reference":
                self._reference(label, body, path)
            else:
                if (kind, label) in self.sections:
                    raise ValueError(f"{path}: section '#{kind} {label}' is defined more than once")
                self.sections[(kind, label)] = self._section(kind, label, body, path)

    def _reference(self, number: str, body: List[str], path: Path) -> None:
        author = date = ""
        text = []
        for ln in body:
            low = ln.strip().lower()
            if low.startswith("@author"):
                author = ln.strip().split(None, 1)[1] if len(ln.split()) > 1 else ""
            elif low.startswith("@date"):
                date = ln.strip().split(None, 1)[1] if len(ln.split()) > 1 else ""
            else:
                text.append(ln.rstrip())
        self.references[(str(path), number)] = Reference(number, "\n".join(text).strip(), author, date, str(path))

    @staticmethod
    def _header(comments: List[str]) -> List[str]:
        for c in reversed(comments):
            if _RULE.match(c) or not c.split():
                continue
            toks = c.split()
            while toks and re.fullmatch(r"(Ver(sion)?|Ref)", toks[0], re.I):
                toks.pop(0)
            return [t for t in toks if t != "#"]
        return []

    def _section(self, kind: str, label: str, body: List[str], path: Path) -> Section:
        sec = Section(kind=kind, label=label, source=str(path))
        data = []
        for ln in body:
            s = ln.strip()
            if not s:
                continue
            if s[0] == "!":
                sec.comments.append(s[1:])
            elif s[0] == ">":
                sec.annotations.append(s[1:].strip())
            elif s[0] == "@" and not s.lower().startswith("@bibtex"):
                w = s[1:].split()
                if w:
                    sec.modifiers.setdefault(w[0], []).append(w[1:])
            else:
                data.append(ln.rstrip())
        if kind in JSON_SECTIONS:
            text = "\n".join(data).strip()
            sec.data = json.loads(text) if text else {}
            return sec
        sch = SCHEMA.get(kind)
        header = self._header(sec.comments)
        if sch is not None and sch["n"] is not None:
            n_key, sym = sch["n"], sch["sym"]
        else:
            n_key = 0
            for t in header:
                if t not in _KEY_TOKENS:
                    break
                n_key += 1
            sym = sch["sym"] if sch is not None else "none"
        sec.key_columns = header[:n_key] if len(header) >= n_key else [f"k{i}" for i in range(n_key)]
        cols = sch["cols"] if sch else None
        text_col = sch.get("text") if sch and cols is not None else None
        if cols is None:
            cols = [(nm, "", None) for nm in header[n_key:]]
        sec.columns = [c[0] for c in cols] + ([text_col] if text_col else [])
        factors = {}
        for mod in sec.modifiers.get("units", []):
            if len(mod) >= 2:
                for c in cols:
                    if c[0] == mod[0] and c[1]:
                        factors[c[0]] = convert_units(1.0, " ".join(mod[1:]), c[1])
        form = sch.get("form") if sch else None
        if form:
            mod = sec.modifier("type")
            in_form = mod[0] if mod else form
            in_units = {m[0].lower(): " ".join(m[1:]) for m in sec.modifiers.get("units", []) if len(m) >= 2}
            form_names = _FORM_PARAMS.get(in_form, ("sigma", "eps"))
            raw = header[n_key:n_key + 2] if len(header) >= n_key + 2 else list(form_names)
            out_names = [c[0] for c in cols[:2]]
            cols, factors = [(nm, "", float) for nm in raw], {}
            sec.columns = out_names
        for ln in data:
            w = ln.split()
            if len(w) < 2 + n_key:
                continue
            key, flipped = canonical_key(sym, w[2:2 + n_key])
            vals = w[2 + n_key:]
            if flipped and sch:
                vals = _flip_values(sch, vals)
            values = {}
            for idx, (name, _unit, ctor) in enumerate(cols):
                if idx >= len(vals):
                    break
                try:
                    v = ctor(vals[idx]) if ctor is not None else _auto(vals[idx])
                except (TypeError, ValueError):
                    v = _auto(vals[idx])
                if name in factors and isinstance(v, float):
                    v *= factors[name]
                values[name] = v
            if text_col:
                values[text_col] = " ".join(vals[len(cols):])
            if form:
                v = list(values.values())
                u1 = in_units.get(form_names[0].lower()) or in_units.get(raw[0].lower())
                u2 = in_units.get(form_names[1].lower()) or in_units.get(raw[1].lower())
                sig, eps = nonbond_to_sigma_eps(in_form, float(v[0]), float(v[1]), u1, u2)
                if form == "rmin-eps":
                    sig *= 2.0 ** (1.0 / 6.0)
                values = {out_names[0]: sig, out_names[1]: eps}
            sec.rows.append(Row(w[0], w[1], key, values, str(path)))
        if form:
            sec.modifiers["type"] = [[form]]
        if form or factors:
            sec.modifiers.pop("units", None)
        return sec

    # ---------------------------------------------------------------------------- resolution
    def forcefield(self, name: Optional[str] = None, version: Optional[str] = None) -> "ForceField":
        """The variant ``name`` (default: the only one, the file's stem, else the first) as of
        ``version`` (default: newest)."""
        if not self.defines:
            raise ValueError(f"{self.path} has no #define section")
        if name is None:
            name = (next(iter(self.defines)) if len(self.defines) == 1 or self.path.stem not in self.defines
                    else self.path.stem)
        if name not in self.defines:
            raise KeyError(f"{self.path} does not define {name!r}; available: {self.forcefields}")
        want = parse_version(version) if version is not None else None
        chosen: Dict[str, tuple] = {}
        for ver, _ref, form, labels in self.defines[name]:
            vk = parse_version(ver)
            if want is not None and vk > want:
                continue
            if form not in chosen or vk >= chosen[form][0]:
                chosen[form] = (vk, labels)
        ff = ForceField(name, self, version)
        for form, (_vk, labels) in chosen.items():
            merged, used, mods, notes = {}, [], {}, []
            for label in labels:
                optional = label.endswith(":optional")
                lab = label[:-9] if optional else label
                sec = self.sections.get((form, lab))
                if sec is None:
                    if optional:
                        continue
                    raise KeyError(f"{self.path}: force field {name!r} needs section '#{form} {lab}'")
                used.append(lab)
                mods.update(sec.modifiers)
                notes = notes or list(sec.annotations)
                if sec.kind in JSON_SECTIONS:
                    merged.update(_latest_json(sec.data, want))
                    continue
                for row in sec.rows:
                    if want is not None and row.version_key > want:
                        continue
                    cur = merged.get(row.key)
                    if cur is None or row.version_key >= cur.version_key:
                        merged[row.key] = row
            ff.sections[form], ff.labels[form], ff.modifiers[form], ff.annotations[form] = merged, used, mods, notes
            cols = next((self.sections[(form, lab)].columns for lab in used if (form, lab) in self.sections), [])
            ff.columns[form] = cols
        ff._finish()
        return ff


def _latest_json(data: dict, want) -> dict:
    out = {}
    for item, versions in (data or {}).items():
        best = None
        for ver, entry in versions.items():
            vk = parse_version(ver)
            if want is not None and vk > want:
                continue
            if best is None or vk >= best[0]:
                best = (vk, ver, entry)
        if best is not None:
            e = dict(best[2])
            e.setdefault("version", best[1])
            out[item] = e
    return out


class ForceField:
    """One resolved variant: ``sections[form] = {key: Row}`` plus typed lookups."""

    def __init__(self, name: str, file: FrcFile, version: Optional[str]):
        self.name, self.file, self.version = name, file, version
        self.sections: Dict[str, dict] = {}
        self.labels: Dict[str, list] = {}
        self.modifiers: Dict[str, dict] = {}
        self.annotations: Dict[str, list] = {}
        self.columns: Dict[str, list] = {}
        self.templates, self.fragments, self.metadata = {}, {}, {}
        self._equiv: dict = {}

    def _finish(self) -> None:
        self.templates = dict(self.sections.pop("templates", {}))
        self.fragments = dict(self.sections.pop("fragments", {}))
        self.metadata = {k[0]: r.values.get("Value") for k, r in self.sections.get("metadata", {}).items()}
        self._equiv = {k[0]: r.values for k, r in self.sections.get("equivalence", {}).items()}

    @property
    def ff_form(self) -> str:
        return str(self.metadata.get("ff_form", ""))

    def kinds_of(self, term: str) -> List[str]:
        return [k for k in self.sections if SCHEMA.get(k, {}).get("cls") == term]

    @property
    def atom_types(self) -> Dict[str, dict]:
        return {k[0]: r.values for k, r in self.sections.get("atom_types", {}).items()}

    def rows(self, kind: str) -> dict:
        return self.sections.get(kind, {})

    def references_used(self) -> List[Reference]:
        seen, out = set(), []
        for rows in self.sections.values():
            for row in rows.values():
                if not isinstance(row, Row) or (row.source, row.reference) in seen:
                    continue
                seen.add((row.source, row.reference))
                ref = self.file.references.get((row.source, row.reference))
                if ref is not None:
                    out.append(ref)
        return out

    def equivalent(self, atom_type: str, term: str) -> str:
        col = {"nonbond": "NonB", "bond": "Bond", "angle": "Angle", "torsion": "Torsion", "oop": "OOP"}[term]
        e = self._equiv.get(atom_type)
        return str(e[col]) if e and col in e else atom_type

    def charge(self, atom_type: str) -> float:
        rows = self.sections.get("charges", {})
        for t in (atom_type, self.equivalent(atom_type, "nonbond")):
            if (t,) in rows:
                return float(rows[(t,)].values["Q"])
        return 0.0

    def nonbond(self, atom_type: str, kind: str = "nonbond(12-6)") -> Optional[Tuple[float, float]]:
        rows = self.sections.get(kind, {})
        row = None
        for t in (atom_type, self.equivalent(atom_type, "nonbond"), WILDCARD):
            row = rows.get((t,))
            if row is not None:
                break
        if row is None or len(row.values) < 2:
            return None
        v = list(row.values.values())
        return float(v[0]), float(v[1])

    def combination(self, kind: str = "nonbond(12-6)") -> str:
        m = self.modifiers.get(kind, {}).get("combination")
        return m[0][0] if m else "geometric"

    def _lookup(self, term: str, sym: str, atoms: Sequence[str], patterns):
        eq = tuple(self.equivalent(a, "oop" if term == "out-of-plane" else term) for a in atoms)
        for cand in (tuple(atoms), eq):
            for kind in self.kinds_of(term):
                rows = self.sections[kind]
                for pat in patterns(cand):
                    key, _ = canonical_key(sym, pat)
                    if key in rows:
                        return kind, key, rows[key]
        return None

    def bond(self, i: str, j: str):
        return self._lookup("bond", "like_bond", (i, j), lambda a: [a])

    def angle(self, i: str, j: str, k: str):
        return self._lookup("angle", "like_angle", (i, j, k), lambda a: [a, (WILDCARD, a[1], WILDCARD)])

    def torsion(self, i: str, j: str, k: str, l: str):
        X = WILDCARD
        return self._lookup("torsion", "like_torsion", (i, j, k, l),
                            lambda a: [a, (X, a[1], a[2], a[3]), (a[0], a[1], a[2], X), (X, a[1], a[2], X)])

    def improper(self, i: str, j: str, k: str, l: str):
        """``k`` central; exact, then one, two and three outer wildcards."""
        X = WILDCARD
        return self._lookup("out-of-plane", "like_improper", (i, j, k, l),
                            lambda a: [a, (X, a[1], a[2], a[3]), (a[0], X, a[2], a[3]), (a[0], a[1], a[2], X),
                                       (X, X, a[2], a[3]), (X, a[1], a[2], X), (a[0], X, a[2], X), (X, X, a[2], X)])


def read_frc(path: Union[str, Path], include_dirs: Sequence[Union[str, Path]] = ()) -> FrcFile:
    return FrcFile(path, include_dirs)


def find_forcefield(spec: str) -> Tuple[Path, Optional[str]]:
    """``(file, variant)`` of a spec: a path (``file.frc`` or ``file.frc:variant``) or the name of a
    shipped file or of a variant defined in one."""
    path, _, variant = str(spec).partition(":") if not Path(spec).is_file() else (spec, "", "")
    if Path(path).is_file():
        return Path(path), variant or None
    cand = DATA_DIR / (path if path.endswith(".frc") else path + ".frc")
    if cand.is_file():
        return cand, variant or None
    for f in sorted(DATA_DIR.glob("*.frc")):
        text = f.read_text(encoding="utf-8", errors="ignore")
        if re.search(rf"^#define\s+{re.escape(spec)}\s*$", text, re.M):
            return f, spec
    raise FileNotFoundError(f"no force field {spec!r} (a .frc path or one of the shipped variants)")


def read_forcefield(spec: str, version: Optional[str] = None) -> ForceField:
    path, variant = find_forcefield(spec)
    return FrcFile(path).forcefield(variant, version)
