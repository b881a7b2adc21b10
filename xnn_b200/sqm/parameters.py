"""NDDO parameter sets and the element data of the MNDO-family methods.

Parameter sets are read and written in the text format MOPAC reads with its
``EXTERNAL=`` keyword (reference ``sqmnn/common/parameters.py:1-30``): one value
per line, ``NAME  Symbol  value`` for an element, ``ALPB_Y  X  value`` /
``XFAC_Y  X  value`` for the diatomic core-core terms of the pair X-Y and
``PARn  value`` for the method's global constants; ``*`` starts a comment and
``END`` (or a blank line) closes the list. A file written here is read back
exactly.

The published PM3 values are MOPAC's data and are not shipped with this
package: a named set (``"pm3"``) is looked up as ``<name>.txt`` in the folder
named by ``XNN_B200_NDDO_DIR``; any other set is given as a path.

Element data (reference ``sqmnn/common/elements.py``): the valence occupations
of the isolated atoms, the principal quantum numbers of the valence shells, the
period that sets the multipole charge separations and the experimental heats of
formation of the gaseous atoms (kcal/mol), for the ``sp`` main-group elements
(H, Li-F, Na-Cl, K, Ca, Ga-Br, Rb, Sr, In-I).
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, Tuple, Union

from ..data.elements import ATOMIC_NUMBERS, SYMBOLS

ELEMENT_KEYS = ("USS", "UPP", "UDD", "ZS", "ZP", "ZD", "BETAS", "BETAP", "BETAD", "GSS", "GSP", "GPP", "GP2",
                "HSP", "F0SD", "G2SD", "POC", "ALP", "ZSN", "ZPN", "ZDN")
GAUSSIAN_KEYS = tuple(f"FN{i}{k}" for k in range(1, 5) for i in range(1, 4))
PAIR_KEYS = ("ALPB", "XFAC")

# experimental heats of formation of the gaseous atoms, kcal/mol (the values MOPAC uses)
ATOM_HEAT = {1: 52.102, 3: 38.41, 4: 76.96, 5: 135.7, 6: 170.89, 7: 113.0, 8: 59.559, 9: 18.89,
             11: 25.65, 12: 35.0, 13: 79.49, 14: 108.39, 15: 75.57, 16: 66.4, 17: 28.99, 19: 21.42, 20: 42.6,
             31: 65.4, 32: 89.5, 33: 72.3, 34: 54.3, 35: 26.74, 37: 19.6, 38: 39.1,
             49: 58.0, 50: 72.2, 51: 63.2, 52: 47.0, 53: 25.517}
SUPPORTED = frozenset(ATOM_HEAT)


def period(z: int) -> int:
    """Row of the periodic table."""
    for row, last in enumerate((2, 10, 18, 36, 54, 86), start=1):
        if z <= last:
            return row
    raise ValueError(f"no period for Z={z}")


def valence_occupation(z: int) -> Tuple[int, int]:
    """``(s, p)`` electrons of the isolated main-group atom."""
    if z not in SUPPORTED:
        raise ValueError(f"element Z={z} is not an sp main-group element of this NDDO implementation")
    if z == 1:
        return 1, 0
    first = {2: 3, 3: 11, 4: 19, 5: 37}[period(z)]
    if z - first < 2:                          # s block
        return z - first + 1, 0
    # the p block starts after the s block, and after the ten d elements from period 4 on
    p_start = first + 2 + (10 if period(z) >= 4 else 0)
    return 2, z - p_start + 1


def principal_quantum_number(z: int) -> int:
    """Principal quantum number of the valence ``s`` and ``p`` Slater orbitals."""
    return period(z)


@dataclass
class NDDOParameters:
    """The parameters of one NDDO method: ``elements`` ``{Z: {NAME: value}}``, ``pairs``
    ``{(Z_high, Z_low): {"ALPB"|"XFAC": value}}`` and ``globals`` ``{n: PARn}``; absent values read as 0."""

    name: str = ""
    elements: Dict[int, Dict[str, float]] = field(default_factory=dict)
    pairs: Dict[Tuple[int, int], Dict[str, float]] = field(default_factory=dict)
    globals: Dict[int, float] = field(default_factory=dict)

    def value(self, z: int, key: str) -> float:
        return float(self.elements.get(int(z), {}).get(key, 0.0))

    def pair_value(self, z1: int, z2: int, key: str) -> float:
        return float(self.pairs.get((max(z1, z2), min(z1, z2)), {}).get(key, 0.0))

    @property
    def atomic_numbers(self) -> Tuple[int, ...]:
        return tuple(sorted(z for z, v in self.elements.items() if v.get("ZS", 0.0) > 0.0 or v.get("GSS", 0.0) > 0.0))


def _parse_line(out: NDDOParameters, tokens) -> bool:
    key = tokens[0].upper()
    if re.fullmatch(r"PAR\d+", key):
        out.globals[int(key[3:])] = float(tokens[1])
        return True
    m = re.fullmatch(r"(ALPB|XFAC)_([A-Za-z]{1,2})", key)
    if m:
        za, zb = ATOMIC_NUMBERS[tokens[1].capitalize()], ATOMIC_NUMBERS[m.group(2).capitalize()]
        out.pairs.setdefault((max(za, zb), min(za, zb)), {})[m.group(1)] = float(tokens[2])
        return True
    if key in ELEMENT_KEYS or key in GAUSSIAN_KEYS:
        out.elements.setdefault(ATOMIC_NUMBERS[tokens[1].capitalize()], {})[key] = float(tokens[2])
        return True
    return False


def load_parameters(source: Union[str, Path, NDDOParameters]) -> NDDOParameters:
    """A parameter set from an ``EXTERNAL`` file, a named set in ``XNN_B200_NDDO_DIR`` or an object."""
    if isinstance(source, NDDOParameters):
        return source
    path = Path(source).expanduser()
    if not path.exists():
        folder = os.environ.get("XNN_B200_NDDO_DIR")
        named = Path(folder) / f"{str(source).lower()}.txt" if folder else None
        if named is None or not named.exists():
            raise FileNotFoundError(
                f"no NDDO parameter file {source!r}: the published sets are MOPAC's data and are not shipped; "
                "give a MOPAC EXTERNAL file, or put <name>.txt in the folder named by XNN_B200_NDDO_DIR")
        path = named
    out = NDDOParameters(name=path.stem)
    for lineno, raw in enumerate(path.read_text().splitlines(), start=1):
        line = raw.strip()
        if line.startswith("*"):
            continue
        if not line or line.upper().startswith("END"):
            break
        try:
            ok = _parse_line(out, line.split())
        except (IndexError, KeyError, ValueError) as exc:
            raise ValueError(f"{path}:{lineno}: cannot read {raw!r}") from exc
        if not ok:
            raise ValueError(f"{path}:{lineno}: unknown parameter {line.split()[0]!r}")
    return out


def save_parameters(params: NDDOParameters, path: Union[str, Path], comment: str = "") -> Path:
    """Write ``params`` as an ``EXTERNAL`` file (values in ``repr`` form, so they read back exactly)."""
    rows = [f"* {c}" for c in comment.splitlines()]
    for z in sorted(params.elements):
        for key in ELEMENT_KEYS + GAUSSIAN_KEYS:
            v = params.elements[z].get(key, 0.0)
            if v != 0.0:
                rows.append(f"{key:<8s}{SYMBOLS[z]:<4s}{v!r:>24s}")
    for (zh, zl), vals in sorted(params.pairs.items()):
        for key in PAIR_KEYS:
            if vals.get(key, 0.0) != 0.0:
                rows.append(f"{key + '_' + SYMBOLS[zl]:<8s}{SYMBOLS[zh]:<4s}{vals[key]!r:>24s}")
    for n in sorted(params.globals):
        if params.globals[n] != 0.0:
            rows.append(f"PAR{n:<5d}{'':4s}{params.globals[n]!r:>24s}")
    rows.append("END")
    path = Path(path)
    path.write_text("\n".join(rows) + "\n")
    return path
