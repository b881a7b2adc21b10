"""AMOEBA parameter sets: a reader of Tinker ``.prm`` files and the AMOEBA water model.

A parameter set holds, per atom type, its class, element, mass, permanent multipole (charge, dipole
and traceless quadrupole in a local frame fixed by up to three neighbouring atom types) and
polarizability (with its Thole damping and polarization-group partners); per atom class the buffered
14-7 van der Waals size, depth and hydrogen reduction factor; per class tuple the valence terms
(quartic bonds, sextic angles, in-plane angles, Urey-Bradley, stretch-bend, Allinger out-of-plane
bends, three-term torsions); and the global coefficients and nonbonded scale factors.

Tinker's keyword grammar is the interchange format of AMOEBA parameters (``atom``, ``vdw``, ``bond``,
``angle``, ``anglep``, ``ureybrad``, ``strbnd``, ``opbend``, ``torsion``, ``multipole`` over five
lines, ``polarize`` and the scalar keywords); :func:`read_prm` parses it. Units are Tinker's: kcal/mol,
Angstrom, degrees, multipoles in e, e bohr and e bohr^2 (as written in the files; quadrupoles are
the traceless Buckingham moments), polarizabilities in A^3.

``AMOEBA_WATER_2003`` is the water model of Ren and Ponder (J. Phys. Chem. B 107, 5933 (2003),
Table 1). Parity: the reference's AMOEBA library reader (``src/xnn/ffnn/models/amoebalib.py``) and
its shipped ``amoeba-water-2003`` set.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Tuple, Union

#: Tinker's keywords that this reader understands but that no term here evaluates
UNSUPPORTED = ("pitors", "tortors", "chgtrn", "repulsion", "dispersion", "chgflx", "bndflx", "angflx")


@dataclass
class MultipoleDef:
    """One ``multipole`` entry: frame-defining neighbour types (signed as in Tinker; 0 = none) and
    the moments in the local frame (e, e bohr, e bohr^2)."""
    z: int
    x: int
    y: int
    q: float
    d: Tuple[float, float, float]
    Q: Tuple[Tuple[float, float, float], ...]

    @property
    def frame(self) -> str:
        """Tinker's frame kinds: ``none``, ``z-only``, ``z-then-x``, ``bisector``, ``z-bisect``, ``3-fold``."""
        if self.z == 0:
            return "none"
        if self.x == 0:
            return "z-only"
        kind = "z-then-x" if (self.z > 0 and self.x > 0) else "bisector"
        if self.x < 0 and self.y < 0:
            kind = "3-fold" if self.z < 0 else "z-bisect"
        return kind


@dataclass
class AmoebaParameters:
    name: str = "amoeba"
    types: Dict[int, Tuple[int, str, int, float]] = field(default_factory=dict)   # type: (class, symbol, Z, mass)
    vdw: Dict[int, Tuple[float, float, float]] = field(default_factory=dict)      # class: (rmin, eps, reduction)
    bonds: Dict[Tuple[int, int], Tuple[float, float]] = field(default_factory=dict)
    angles: Dict[Tuple[int, int, int], Tuple[float, Tuple[float, ...], bool]] = field(default_factory=dict)
    ureybrad: Dict[Tuple[int, int, int], Tuple[float, float]] = field(default_factory=dict)
    strbnd: Dict[Tuple[int, int, int], Tuple[float, float]] = field(default_factory=dict)
    opbend: Dict[Tuple[int, int, int, int], float] = field(default_factory=dict)
    torsions: Dict[Tuple[int, int, int, int], List[Tuple[float, float, int]]] = field(default_factory=dict)
    multipoles: Dict[int, List[MultipoleDef]] = field(default_factory=dict)
    polarize: Dict[int, Tuple[float, float, Tuple[int, ...]]] = field(default_factory=dict)
    scalars: Dict[str, object] = field(default_factory=dict)
    unsupported: List[str] = field(default_factory=list)
    #: the Tinker text the set was read from (written back by the Tinker input writer)
    source_text: Optional[str] = None

    # ------------------------------------------------------------------ scalar access
    def get(self, key: str, default):
        v = self.scalars.get(key.lower(), default)
        if isinstance(default, float):
            return float(v)
        return v

    def scale(self, kind: str, sep: int) -> float:
        """Nonbonded scale factor ``<kind>-1<sep>-scale`` (``sep`` 2..5; 1 for the other kinds
        of separation) with Tinker's defaults for AMOEBA."""
        defaults = {"vdw": (0.0, 0.0, 1.0, 1.0), "mpole": (0.0, 0.0, 0.4, 0.8), "polar": (0.0, 0.0, 1.0, 1.0)}
        base = defaults.get(kind, (1.0, 1.0, 1.0, 1.0))
        return self.get(f"{kind}-1{sep}-scale", float(base[sep - 2]))

    def group_scale(self, kind: str, sep: int) -> float:
        """``direct-1<sep>-scale`` / ``mutual-1<sep>-scale``: by polarization-group separation
        (``sep`` 1 = same group, 2 = bonded groups, ...)."""
        base = {"direct": (0.0, 1.0, 1.0, 1.0), "mutual": (1.0, 1.0, 1.0, 1.0)}[kind]
        return self.get(f"{kind}-1{sep}-scale", float(base[sep - 1]) if sep <= 4 else 1.0)

    # ------------------------------------------------------------------ lookups
    def type_class(self, t: int) -> int:
        return self.types[t][0]

    def bond(self, a: int, b: int):
        return self.bonds.get((min(a, b), max(a, b)))

    def angle(self, a: int, b: int, c: int):
        return self.angles.get((min(a, c), b, max(a, c)))

    def urey(self, a: int, b: int, c: int):
        return self.ureybrad.get((min(a, c), b, max(a, c)))

    def stretch_bend(self, a: int, b: int, c: int):
        """``(k_ab, k_cb)`` for the angle a-b-c (the file's order may be either way round)."""
        if (a, b, c) in self.strbnd:
            return self.strbnd[(a, b, c)]
        if (c, b, a) in self.strbnd:
            k1, k2 = self.strbnd[(c, b, a)]
            return k2, k1
        return None

    def torsion(self, a: int, b: int, c: int, d: int):
        key = (a, b, c, d) if (b, a) <= (c, d) else (d, c, b, a)
        if key in self.torsions:
            return self.torsions[key]
        for k in ((a, b, c, d), (d, c, b, a)):
            if k in self.torsions:
                return self.torsions[k]
        return None

    def out_of_plane(self, d: int, b: int, a: int, c: int) -> Optional[float]:
        """Allinger out-of-plane constant of atom class ``d`` bent out of the plane of centre ``b``
        with ``a``, ``c`` (0 matches any class)."""
        for key in ((d, b, a, c), (d, b, c, a), (d, b, a, 0), (d, b, c, 0), (d, b, 0, 0)):
            if key in self.opbend:
                return self.opbend[key]
        return None


def _floats(tokens) -> List[float]:
    return [float(t) for t in tokens]


def _is_int(tok: str) -> bool:
    try:
        int(tok)
        return True
    except ValueError:
        return False


def parse_prm(text: str, name: str = "amoeba") -> AmoebaParameters:
    """Parameters from the text of a Tinker ``.prm`` file."""
    p = AmoebaParameters(name=name)
    lines = [ln.split("#")[0].rstrip() for ln in text.splitlines()]
    k = 0
    while k < len(lines):
        ln = lines[k].strip()
        k += 1
        if not ln:
            continue
        tok = ln.replace('"', ' " ').split()
        key = tok[0].lower()
        if key == "atom":
            # atom type class symbol "description" Z mass valence
            q1 = ln.index('"')
            q2 = ln.index('"', q1 + 1)
            head = ln[:q1].split()
            tail = ln[q2 + 1:].split()
            p.types[int(head[1])] = (int(head[2]), head[3], int(tail[0]), float(tail[1]))
        elif key == "vdw":
            v = _floats(tok[2:])
            p.vdw[int(tok[1])] = (v[0], v[1], v[2] if len(v) > 2 else 1.0)
        elif key == "bond":
            a, b = int(tok[1]), int(tok[2])
            p.bonds[(min(a, b), max(a, b))] = (float(tok[3]), float(tok[4]))
        elif key in ("angle", "anglep"):
            a, b, c = int(tok[1]), int(tok[2]), int(tok[3])
            v = _floats(tok[4:])
            p.angles[(min(a, c), b, max(a, c))] = (v[0], tuple(v[1:]), key == "anglep")
        elif key == "ureybrad":
            a, b, c = int(tok[1]), int(tok[2]), int(tok[3])
            p.ureybrad[(min(a, c), b, max(a, c))] = (float(tok[4]), float(tok[5]))
        elif key == "strbnd":
            p.strbnd[(int(tok[1]), int(tok[2]), int(tok[3]))] = (float(tok[4]), float(tok[5]))
        elif key == "opbend":
            p.opbend[tuple(int(t) for t in tok[1:5])] = float(tok[5])
        elif key == "torsion":
            cls = tuple(int(t) for t in tok[1:5])
            v = tok[5:]
            terms = [(float(v[i]), float(v[i + 1]), int(v[i + 2])) for i in range(0, len(v) - 2, 3)]
            p.torsions[cls] = terms
        elif key == "multipole":
            ints = [int(t) for t in tok[1:-1] if _is_int(t)]
            t_, frame = ints[0], ints[1:] + [0] * (3 - len(ints[1:]))
            q = float(tok[-1])
            rows = []
            while len(rows) < 4 and k < len(lines):
                s = lines[k].strip()
                k += 1
                if s:
                    rows.append(_floats(s.split()))
            d = tuple(rows[0])
            qxx, (qxy, qyy), (qxz, qyz, qzz) = rows[1][0], rows[2], rows[3]
            Q = ((qxx, qxy, qxz), (qxy, qyy, qyz), (qxz, qyz, qzz))
            p.multipoles.setdefault(t_, []).append(MultipoleDef(frame[0], frame[1], frame[2], q, d, Q))
        elif key == "polarize":
            v = tok[2:]
            p.polarize[int(tok[1])] = (float(v[0]), float(v[1]), tuple(int(x) for x in v[2:]))
        elif key in UNSUPPORTED:
            if key not in p.unsupported:
                p.unsupported.append(key)
        elif len(tok) >= 2 and not _is_int(tok[1]):
            val = tok[1]
            try:
                val = float(val)
            except ValueError:
                val = val.upper()
            p.scalars[key] = val
        elif len(tok) == 1:
            p.scalars[key] = True
    return p


def read_prm(path: Union[str, Path]) -> AmoebaParameters:
    path = Path(path)
    text = path.read_text()
    p = parse_prm(text, name=path.stem)
    p.source_text = text
    return p


#: AMOEBA water (Ren and Ponder 2003, Table 1): Tinker types 1 (O) and 2 (H)
AMOEBA_WATER_2003_PRM = """
forcefield              AMOEBA-WATER-2003
bond-cubic              -2.55
bond-quartic            3.793125
angle-cubic             -0.014
angle-quartic           0.000056
angle-pentic            -0.0000007
angle-sextic            0.000000022
opbendtype              ALLINGER
opbend-cubic            -0.014
opbend-quartic          0.000056
opbend-pentic           -0.0000007
opbend-sextic           0.000000022
torsionunit             0.5
vdwtype                 BUFFERED-14-7
radiusrule              CUBIC-MEAN
radiustype              R-MIN
radiussize              DIAMETER
epsilonrule             HHG
dielectric              1.0
polarization            MUTUAL
vdw-12-scale            0.0
vdw-13-scale            0.0
vdw-14-scale            1.0
vdw-15-scale            1.0
mpole-12-scale          0.0
mpole-13-scale          0.0
mpole-14-scale          0.4
mpole-15-scale          0.8
polar-12-scale          0.0
polar-13-scale          0.0
polar-14-scale          1.0
polar-15-scale          1.0
polar-14-intra          0.5
direct-11-scale         0.0
direct-12-scale         1.0
direct-13-scale         1.0
direct-14-scale         1.0
mutual-11-scale         1.0
mutual-12-scale         1.0
mutual-13-scale         1.0
mutual-14-scale         1.0

atom          1    1    O     "AMOEBA Water O"    8    15.995    2
atom          2    2    H     "AMOEBA Water H"    1     1.008    1

vdw           1               3.4050     0.1100
vdw           2               2.6550     0.0135      0.910

bond          1    2          529.60     0.9572
angle         2    1    2      34.05     108.50
ureybrad      2    1    2      38.25     1.5537

multipole     1   -2   -2              -0.51966
                                        0.00000    0.00000    0.14279
                                        0.37928
                                        0.00000   -0.41809
                                        0.00000    0.00000    0.03881
multipole     2    1    2               0.25983
                                       -0.03859    0.00000   -0.05818
                                       -0.03673
                                        0.00000   -0.10739
                                       -0.00203    0.00000    0.14412

polarize      1          0.837     0.390     2
polarize      2          0.496     0.390     1
"""


def amoeba_water_2003() -> AmoebaParameters:
    p = parse_prm(AMOEBA_WATER_2003_PRM, name="amoeba-water-2003")
    p.source_text = AMOEBA_WATER_2003_PRM
    return p


def load_parameters(source) -> AmoebaParameters:
    """A parameter set from a shipped name (``"amoeba-water-2003"``), a ``.prm`` path or an instance."""
    if isinstance(source, AmoebaParameters):
        return source
    if isinstance(source, str) and source.lower() in ("amoeba-water-2003", "water03", "amoeba_water_2003"):
        return amoeba_water_2003()
    return read_prm(source)


# ----------------------------------------------------------------------------- Tinker inputs
def write_tinker_xyz(path: Union[str, Path], positions, types, bonds, symbols, title: str = "xnn_b200",
                     cell=None) -> Path:
    """A Tinker ``.xyz`` file: atom count and title, the box (lengths and angles) when ``cell`` is
    given, then per atom its index, symbol, position (A), Tinker type and bonded neighbours
    (1-based)."""
    import math as _m

    import numpy as np
    pos = np.asarray(positions, dtype=float)
    n = pos.shape[0]
    nbr = [[] for _ in range(n)]
    for i, j in bonds:
        nbr[int(i)].append(int(j) + 1)
        nbr[int(j)].append(int(i) + 1)
    lines = [f"{n:6d}  {title}"]
    if cell is not None:
        c = np.asarray(cell, dtype=float)
        a, b, cc = (float(np.linalg.norm(v)) for v in c)
        ang = lambda u, v: _m.degrees(_m.acos(float(np.dot(u, v)) / (np.linalg.norm(u) * np.linalg.norm(v))))  # noqa
        lines.append(f"{a:12.6f}{b:12.6f}{cc:12.6f}{ang(c[1], c[2]):12.6f}{ang(c[0], c[2]):12.6f}{ang(c[0], c[1]):12.6f}")
    for k in range(n):
        conn = "".join(f"{x:6d}" for x in sorted(nbr[k]))
        lines.append(f"{k + 1:6d}  {symbols[k]:<3s}{pos[k, 0]:12.6f}{pos[k, 1]:12.6f}{pos[k, 2]:12.6f}"
                     f"{int(types[k]):6d}{conn}")
    p = Path(path)
    p.write_text("\n".join(lines) + "\n")
    return p


def read_tinker_xyz(path: Union[str, Path]):
    """``(positions (n, 3), types, bonds, symbols, cell or None)`` of a Tinker ``.xyz`` file."""
    import math as _m

    import numpy as np
    lines = [ln for ln in Path(path).read_text().splitlines()]
    n = int(lines[0].split()[0])
    body = lines[1:]
    cell = None
    first = body[0].split()
    if len(first) == 6 and all(_is_float(x) for x in first):
        a, b, c, al, be, ga = (float(x) for x in first)
        al, be, ga = (_m.radians(x) for x in (al, be, ga))
        cx = _m.cos(be)
        cy = (_m.cos(al) - _m.cos(be) * _m.cos(ga)) / _m.sin(ga)
        cell = np.array([[a, 0, 0], [b * _m.cos(ga), b * _m.sin(ga), 0],
                         [c * cx, c * cy, c * _m.sqrt(max(0.0, 1 - cx * cx - cy * cy))]])
        body = body[1:]
    pos, types, syms, bonds = np.zeros((n, 3)), [], [], set()
    for k in range(n):
        f = body[k].split()
        syms.append(f[1])
        pos[k] = [float(x) for x in f[2:5]]
        types.append(int(f[5]))
        for j in f[6:]:
            a, b = k, int(j) - 1
            bonds.add((min(a, b), max(a, b)))
    return pos, types, sorted(bonds), syms, cell


def _is_float(x: str) -> bool:
    try:
        float(x)
        return True
    except ValueError:
        return False


def write_tinker_key(path: Union[str, Path], prm_name: str, cell=None, cutoff: float = 9.0,
                     ewald_cutoff: float = 7.0, polar_eps: float = 1e-8) -> Path:
    """A Tinker ``.key`` file naming the parameter file; Ewald and cutoffs for a periodic box."""
    lines = [f"parameters  {prm_name}", "verbose", f"polar-eps  {polar_eps:g}"]
    if cell is not None:
        lines += ["ewald", f"ewald-cutoff  {ewald_cutoff:g}", f"vdw-cutoff  {cutoff:g}", "neighbor-list"]
    p = Path(path)
    p.write_text("\n".join(lines) + "\n")
    return p
