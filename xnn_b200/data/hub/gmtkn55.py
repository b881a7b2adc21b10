"""GMTKN55 (Goerigk et al., PCCP 19, 32184, 2017): 55 sets of main-group reaction energies,
barrier heights and noncovalent interactions with high-level references (kcal/mol).

Read from the distribution repository archive: per set a folder with one sub-folder per species
(``struc.xyz``, ``.CHRG``, ``.UHF``, optionally ``PBEh-3c/orca.out``) and the reference file
``.res`` whose ``$tmer`` lines list species (``a{1,2}b`` expands to ``a1b a2b``), ``x``, the
stoichiometric coefficients, ``$w`` and the reference energy. ``split``: ``structures`` (alias
``all``), ``reactions`` or None (both, the input of
:meth:`xnn_b200.train.reactions.ReactionSet.from_gmtkn55`). The set / category table, the archive
versions and the species-name corrections follow the reference's loader
(``src/xnn/common/data/hub/gmtkn55.py``).
"""
from __future__ import annotations

import re
import zipfile
from pathlib import Path
from typing import Iterable, List, Optional, Sequence, Tuple, Union

import numpy as np

from ..elements import ATOMIC_NUMBERS
from .base import DatasetBuilder, register_dataset
from .download import UNITS, fetch

URL = "https://github.com/grimme-lab/GMTKN55/archive/{commit}.zip"
VERSIONS = {"v1": ("8d485b37a1ca8837e395042671ca5ba4e0714691", "1c83333b9009045e83c7cf3a6ccdf5cc"),
            "v2": ("ccabc16c8c4677fc60c19870ae96ac25405844a2", "5c92f8fc05e350bb35cf9c5d82d317ce")}
CATEGORIES = {
    "small_reactions": ("W4-11", "G21EA", "G21IP", "DIPCS10", "PA26", "SIE4x4", "ALKBDE10", "YBDE18", "AL2X6",
                        "HEAVYSB11", "NBPRC", "ALK8", "RC21", "G2RC", "BH76RC", "FH51", "TAUT15", "DC13"),
    "large_reactions": ("MB16-43", "DARC", "RSE43", "BSR36", "CDIE20", "ISO34", "ISOL24", "C60ISO", "PArel"),
    "barrier_heights": ("BH76", "BHPERI", "BHDIV10", "INV24", "BHROT27", "PX13", "WCPT18"),
    "intermolecular_nci": ("RG18", "ADIM6", "S22", "S66", "HEAVY28", "WATER27", "CARBHB12", "PNICO23", "HAL59",
                           "AHB21", "CHB6", "IL16"),
    "intramolecular_nci": ("IDISP", "ICONF", "ACONF", "Amino20x4", "PCONF21", "MCONF", "SCONF", "UPU23",
                           "BUT14DIOL"),
}
SUBSETS = tuple(s for sets in CATEGORIES.values() for s in sets)
CATEGORY_OF = {s: c for c, sets in CATEGORIES.items() for s in sets}
_FOLDER = {"BH76RC": "BH76"}                     # BH76RC shares BH76's species, with its own .resRC
_RES_FILE = {"BH76RC": ".resRC"}
# species renamed between the repository versions (the v2 .res of WATER27 names a few differently)
_SPECIES_FIXES = {"v2": {"WATER27": (("H1O", "H2O"), ("H2Op", "H3Op"), ("OHmH1O", "OHmH2O"))}}
_KEEP = ("/struc.xyz", "/.CHRG", "/.UHF", "/.res", "/.resRC", "/PBEh-3c/orca.out")


def _expand(token: str) -> List[str]:
    name = token.split("/")[0]
    m = re.fullmatch(r"([^{}]*)\{([^{}]*)\}([^{}]*)", name)
    if m:
        return [m.group(1) + part + m.group(3) for part in m.group(2).split(",")]
    if "{" in name or "}" in name:
        raise ValueError(f"cannot expand species token {token!r}")
    return [name]


def parse_reactions(text: str) -> List[Tuple[List[str], List[int], float]]:
    """``(species, coefficients, reference kcal/mol)`` of each ``$tmer`` line of a ``.res`` file."""
    out = []
    for raw in text.splitlines():
        tok = raw.split("#", 1)[0].split()
        if len(tok) < 5 or tok[0] not in ("$tmer", "tmer2++") or "x" not in tok or "$w" not in tok:
            continue
        ix, iw = tok.index("x"), tok.index("$w")
        species = [s for t in tok[1:ix] for s in _expand(t)]
        coef = [int(t) for t in tok[ix + 1:iw]]
        if len(species) != len(coef):
            raise ValueError(f"species and coefficients differ in length: {raw!r}")
        tail = []
        for t in tok[iw + 2:]:
            try:
                tail.append(float(t))
            except ValueError:
                break
        if tail and (tail[0] != 0.0 or (len(tail) > 1 and tail[1] != 1.0)):
            raise ValueError(f"unsupported energy offset / error multiplier: {raw!r}")
        out.append((species, coef, float(tok[iw + 1])))
    return out


def _canonical(subset: str) -> str:
    key = subset.strip().lower().replace("_", "-")
    for s in SUBSETS:
        if s.lower() == key:
            return s
    raise ValueError(f"unknown GMTKN55 set {subset!r}; choose from {', '.join(SUBSETS)}")


def _structure(folder: Path, subset: str, name: str) -> dict:
    xyz = folder / "struc.xyz"
    if not xyz.exists():
        raise FileNotFoundError(f"no geometry for species {name!r} of {subset} ({folder})")
    lines = xyz.read_text().splitlines()
    n = int(lines[0].split()[0])
    rows = [line.split() for line in lines[2:2 + n]]
    z = np.array([ATOMIC_NUMBERS[r[0].capitalize()] if not r[0].isdigit() else int(r[0]) for r in rows], dtype=np.int64)
    pos = np.array([[float(v) for v in r[1:4]] for r in rows], dtype=np.float64)

    def integer(p, default=0):
        return int(p.read_text().split()[0]) if p.exists() else default
    d = {"atomic_numbers": z, "pos": pos, "total_charge": float(integer(folder / ".CHRG")),
         "spin_multiplicity": float(integer(folder / ".UHF")) + 1.0, "subset": subset,
         "category": CATEGORY_OF[subset], "name": name}
    orca = folder / "PBEh-3c" / "orca.out"
    if orca.exists():
        e = [float(line.split()[-1]) for line in orca.read_text().splitlines() if "FINAL SINGLE POINT ENERGY" in line]
        if e:
            d["pbeh3c_energy"] = e[-1] * UNITS["hartree_to_ev"]
    return d


class GMTKN55(DatasetBuilder):
    name = "gmtkn55"
    description = ("GMTKN55: 55 sets, 1505 main-group reaction energies, barrier heights and noncovalent "
                   "interactions (kcal/mol references) on 2462 structures.")

    def load(self, *, split: Optional[str] = None, cache_dir: Path, version: str = "v2",
             subsets: Optional[Union[str, Sequence[str]]] = None, elements: Optional[Iterable] = None,
             max_abs_charge: Optional[float] = None, closed_shell: bool = False, **_):
        """Reactions whose species all pass the filters (``elements``, ``max_abs_charge``,
        ``closed_shell``) and the structures they use."""
        if split not in (None, "all", "structures", "reactions"):
            raise ValueError("split must be None, 'structures' ('all') or 'reactions'")
        if version not in VERSIONS:
            raise ValueError(f"version must be one of {sorted(VERSIONS)}")
        names = SUBSETS if subsets is None else [_canonical(s) for s in ([subsets] if isinstance(subsets, str)
                                                                          else subsets)]
        allowed = None if elements is None else {ATOMIC_NUMBERS[e] if isinstance(e, str) else int(e) for e in elements}
        root = self._extracted(Path(cache_dir) / self.name / "raw", version)
        structures, reactions = [], []
        for subset in names:
            folder = root / _FOLDER.get(subset, subset)
            fixes = _SPECIES_FIXES.get(version, {}).get(subset, ())
            cache: dict = {}
            for k, (species, coef, ref) in enumerate(parse_reactions((folder / _RES_FILE.get(subset, ".res"))
                                                                     .read_text()), 1):
                species = [next((right + s[len(wrong):] for wrong, right in fixes if s.startswith(wrong)), s)
                           for s in species]
                for s in species:
                    if s not in cache:
                        cache[s] = _structure(folder / s, subset, s)
                ok = all((allowed is None or set(cache[s]["atomic_numbers"].tolist()) <= allowed)
                         and (max_abs_charge is None or abs(cache[s]["total_charge"]) <= max_abs_charge)
                         and (not closed_shell or cache[s]["spin_multiplicity"] == 1.0) for s in species)
                if ok:
                    reactions.append({"subset": subset, "category": CATEGORY_OF[subset], "index": k,
                                      "species": species, "stoichiometry": coef, "reference": ref})
            used = {s for r in reactions if r["subset"] == subset for s in r["species"]}
            structures.extend(cache[s] for s in cache if s in used)
        out = {"structures": structures, "reactions": reactions}
        return out if split is None else out["structures" if split == "all" else split]

    @staticmethod
    def _extracted(raw: Path, version: str) -> Path:
        root = raw / version
        marker = root / ".extracted"
        if marker.exists():
            return root
        commit, md5 = VERSIONS[version]
        archive = fetch(URL.format(commit=commit), raw / f"GMTKN55-{version}.zip", md5)
        with zipfile.ZipFile(archive) as zf:
            for member in zf.namelist():
                rel = member.split("/", 1)[1] if "/" in member else ""
                if rel and not member.endswith("/") and (member.endswith(_KEEP) or rel in ("README.md", "LICENSE")):
                    dest = root / rel
                    dest.parent.mkdir(parents=True, exist_ok=True)
                    dest.write_bytes(zf.read(member))
        marker.write_text(commit + "\n")
        return root


register_dataset(GMTKN55())
