"""QM9 (Ramakrishnan et al., Sci. Data 1, 140022, 2014): 133,885 GDB-9 molecules (H, C, N, O, F)
with B3LYP/6-31G(2df,p) geometries and 15 properties.

Read from the distribution archive of per-molecule XYZ files, whose second line holds ``gdb
<index>`` and the 15 properties (``A B C mu alpha homo lumo gap r2 zpve U0 U H G Cv``; energies in
hartree) and whose coordinate lines may write exponents as ``*^``. The parsed set is cached as one
``.npz``. The 3,054 molecules that failed the authors' consistency check (the published
``uncharacterized.txt``) are left out by default. Labels and the atomic reference energies of
``U0 / U / H / G`` (published with the set) follow the reference's loader
(``src/xnn/common/data/hub/qm9.py``); splits are a seeded permutation.
"""
from __future__ import annotations

import io
import tarfile
from pathlib import Path
from typing import Dict, Optional, Tuple

import numpy as np

from .base import DatasetBuilder, register_dataset
from .download import UNITS, fetch

XYZ_ARCHIVE = ("https://ndownloader.figshare.com/files/3195389", "ad1ebd51ee7f5b3a6e32e974e5d54012")
UNCHARACTERIZED = ("https://ndownloader.figshare.com/files/3195404", "a361887bacb427b8a0ce7903d92a53b4")
PROPERTIES = ("A", "B", "C", "mu", "alpha", "homo", "lumo", "gap", "r2", "zpve", "U0", "U", "H", "G", "Cv")
ENERGY_PROPERTIES = ("homo", "lumo", "gap", "zpve", "U0", "U", "H", "G")
_Z = {"H": 1, "C": 6, "N": 7, "O": 8, "F": 9}
# free-atom energies (hartree) of the thermochemical labels, as published with QM9
ATOMIC_REFERENCES = {
    "U0": {1: -0.500273, 6: -37.846772, 7: -54.583861, 8: -75.064579, 9: -99.718730},
    "U": {1: -0.498857, 6: -37.845355, 7: -54.582445, 8: -75.063163, 9: -99.717314},
    "H": {1: -0.497912, 6: -37.844411, 7: -54.581501, 8: -75.062219, 9: -99.716370},
    "G": {1: -0.510927, 6: -37.861317, 7: -54.598897, 8: -75.079532, 9: -99.733544},
}


def atomic_energies(label: str = "U0", units: str = "eV") -> Dict[int, float]:
    if label not in ATOMIC_REFERENCES:
        raise ValueError(f"no atomic references for {label!r}; choose from {sorted(ATOMIC_REFERENCES)}")
    f = UNITS["hartree_to_ev"] if units == "eV" else 1.0
    return {z: e * f for z, e in ATOMIC_REFERENCES[label].items()}


def parse_xyz(text: str) -> Tuple[int, np.ndarray, np.ndarray, np.ndarray]:
    """``(index, atomic numbers, positions, 15 properties)`` of one QM9 XYZ file."""
    lines = text.splitlines()
    n = int(lines[0].split()[0])
    head = lines[1].split()
    props = np.array([float(v) for v in head[2:2 + len(PROPERTIES)]], dtype=np.float64)
    z = np.empty(n, dtype=np.int64)
    pos = np.empty((n, 3), dtype=np.float64)
    for k, line in enumerate(lines[2:2 + n]):
        f = line.replace("*^", "e").split()
        z[k], pos[k] = _Z[f[0]], [float(v) for v in f[1:4]]
    return int(head[1]), z, pos, props


def parse_archive(path) -> Dict[str, np.ndarray]:
    """Every ``.xyz`` member of the archive, ordered by molecule index, as flat arrays."""
    mols = []
    with tarfile.open(path, "r:*") as tar:
        for member in tar:
            if member.isfile() and member.name.endswith(".xyz"):
                fh = tar.extractfile(member)
                if fh is not None:
                    mols.append(parse_xyz(io.TextIOWrapper(fh, encoding="utf-8").read()))
    mols.sort(key=lambda m: m[0])
    counts = np.array([len(m[1]) for m in mols], dtype=np.int64)
    return {"index": np.array([m[0] for m in mols], dtype=np.int64),
            "atomic_numbers": np.concatenate([m[1] for m in mols]) if mols else np.zeros(0, np.int64),
            "pos": np.concatenate([m[2] for m in mols]) if mols else np.zeros((0, 3)),
            "properties": np.stack([m[3] for m in mols]) if mols else np.zeros((0, len(PROPERTIES))),
            "offsets": np.concatenate([[0], np.cumsum(counts)])}


def uncharacterized_ids(path) -> np.ndarray:
    ids = {int(f[0]) for f in (line.split() for line in Path(path).read_text().splitlines()) if f and f[0].isdigit()}
    return np.array(sorted(ids), dtype=np.int64)


class QM9(DatasetBuilder):
    name = "qm9"
    description = "QM9: 133,885 GDB-9 molecules (H, C, N, O, F), B3LYP energies and 14 further properties."

    def load(self, *, split: Optional[str] = None, cache_dir: Path, label: str = "U0", units: str = "eV",
             n_train: int = 110000, n_val: int = 10000, n_test: Optional[int] = None, seed: int = 0,
             exclude_uncharacterized: bool = True, return_info: bool = False, **_):
        """Structures ``{"pos", "atomic_numbers", "energy"}`` (``energy`` is the property ``label``,
        energies in eV or hartree); ``split`` ``train`` / ``val`` / ``test`` / ``all`` / None (a
        dict of the three)."""
        if units not in ("eV", "hartree"):
            raise ValueError(f"units must be 'eV' or 'hartree', got {units!r}")
        if label not in PROPERTIES:
            raise ValueError(f"unknown label {label!r}; choose from {PROPERTIES}")
        root = Path(cache_dir) / self.name
        cache = root / "qm9.npz"
        if not cache.exists():
            archive = fetch(XYZ_ARCHIVE[0], root / "raw" / "dsgdb9nsd.xyz.tar.bz2", XYZ_ARCHIVE[1])
            root.mkdir(parents=True, exist_ok=True)
            np.savez(cache, **parse_archive(archive))
        d = np.load(cache)
        index, offsets, pos, z = d["index"], d["offsets"], d["pos"], d["atomic_numbers"]
        keep = np.ones(len(index), dtype=bool)
        if exclude_uncharacterized:
            bad = uncharacterized_ids(fetch(UNCHARACTERIZED[0], root / "raw" / "uncharacterized.txt",
                                            UNCHARACTERIZED[1]))
            keep &= ~np.isin(index, bad)
        scale = np.array([UNITS["hartree_to_ev"] if units == "eV" and p in ENERGY_PROPERTIES else 1.0
                          for p in PROPERTIES])
        props = d["properties"] * scale
        col = PROPERTIES.index(label)

        def build(rows):
            out = []
            for i in rows:
                a, b = offsets[i], offsets[i + 1]
                s = {"pos": pos[a:b].copy(), "atomic_numbers": z[a:b].copy(), "energy": float(props[i, col])}
                if return_info:
                    s["info"] = {"index": int(index[i]), **{k: float(v) for k, v in zip(PROPERTIES, props[i])}}
                out.append(s)
            return out
        rows = np.flatnonzero(keep)
        if split == "all":
            return build(rows)
        perm = rows[np.random.default_rng(seed).permutation(len(rows))]
        splits = {"train": build(np.sort(perm[:n_train])), "val": build(np.sort(perm[n_train:n_train + n_val])),
                  "test": build(np.sort(perm[n_train + n_val:][:n_test]))}
        if split is None:
            return splits
        if split not in splits:
            raise ValueError(f"unknown split {split!r}; use 'train', 'val', 'test', 'all' or None")
        return splits[split]


register_dataset(QM9())
