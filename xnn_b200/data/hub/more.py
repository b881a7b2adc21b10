"""More dataset builders: OC20 S2EF (200K), Materials Project 2018 (MEGNet), and ASE SQLite databases.

* ``oc20_s2ef_200k`` (Chanussot et al., ACS Catal. 11, 6059 (2021), CC BY 4.0): the smallest S2EF
  training split, a tar of xz-compressed ``.extxyz`` frames with one ``.txt`` per file listing each
  frame's system id, frame index and reference energy. ``energy="adsorption"`` (default) stores the
  energy minus that reference; ``"total"`` the DFT energy. Atoms the relaxation held fixed get an
  ``atom_force_weight`` of zero; ``info`` keeps ``tags`` (0 subsurface, 1 surface, 2 adsorbate).
* ``mp_2018`` (Chen et al., Chem. Mater. 31, 3564 (2019), CC BY 4.0): the 69,239 crystals of the
  MEGNet paper (a zipped JSON list; each entry's structure is a P1 CIF) with formation energy per
  atom, band gap and, where computed, bulk / shear moduli (``log10`` in the file).
* ``ase_db``: any ASE SQLite database (``path=``), read with the standard library's ``sqlite3``:
  positions, numbers, cell, pbc, energy, forces, stress, charges, and the key-value pairs in
  ``info``.

Splits are seeded permutations (80 / 10 / 10). Parity: the reference's dataset hub
(``src/xnn/common/data/hub/oc20.py``, ``materials_project.py``, ``_sqlite.py``).
"""
from __future__ import annotations

import io
import json
import lzma
import math
import re
import sqlite3
import tarfile
import zipfile
from pathlib import Path
from typing import Dict, List, Optional

import numpy as np
import torch

from ..elements import ATOMIC_NUMBERS
from ..io import read_extxyz
from .base import DatasetBuilder, register_dataset, select_split
from .download import fetch


def seeded_splits(items: list, seed: int = 0, fractions=(0.8, 0.1)) -> Dict[str, list]:
    perm = np.random.default_rng(seed).permutation(len(items))
    n_tr = int(round(fractions[0] * len(items)))
    n_va = int(round(fractions[1] * len(items)))
    pick = lambda idx: [items[int(k)] for k in idx]  # noqa: E731
    return {"train": pick(perm[:n_tr]), "val": pick(perm[n_tr:n_tr + n_va]), "test": pick(perm[n_tr + n_va:])}


# ----------------------------------------------------------------------------- OC20
OC20_200K = ("https://dl.fbaipublicfiles.com/opencatalystproject/data/s2ef_train_200K.tar",
             "f8d0909c2623a393148435dede7d3a46")


def read_oc20_archive(path, energy: str = "adsorption", max_frames: Optional[int] = None) -> List[dict]:
    """Frames of an S2EF archive: each ``.extxyz.xz`` member with its ``.txt`` references."""
    frames: List[dict] = []
    with tarfile.open(path) as tar:
        members = {m.name: m for m in tar.getmembers() if m.isfile()}
        for name in sorted(n for n in members if n.endswith(".extxyz.xz")):
            base = name[:-len(".extxyz.xz")]
            text = lzma.decompress(tar.extractfile(members[name]).read()).decode()
            txt = members.get(base + ".txt")
            refs = []
            if txt is not None:
                for line in tar.extractfile(txt).read().decode().splitlines():
                    f = [x.strip() for x in line.split(",")]
                    if len(f) >= 3:
                        refs.append((f[0], f[1], float(f[2])))
            tmp = io.StringIO(text)
            parsed = _extxyz_text(tmp.getvalue())
            for k, s in enumerate(parsed):
                if "move_mask" in s:
                    s["atom_force_weight"] = torch.as_tensor(s.pop("move_mask"), dtype=torch.float64)
                sid, frame, ref = refs[k] if k < len(refs) else ("", "", 0.0)
                s["info"] = {"system_id": sid, "frame": frame, "reference_energy": ref,
                             "tags": s.pop("tags", None)}
                if energy == "adsorption" and "energy" in s:
                    s["energy"] = float(s["energy"]) - ref
                frames.append(s)
                if max_frames is not None and len(frames) >= max_frames:
                    return frames
    return frames


def _extxyz_text(text: str) -> List[dict]:
    """:func:`~xnn_b200.data.io.read_extxyz` on text, keeping the OC20 columns ``move_mask`` and
    ``tags``."""
    import tempfile
    with tempfile.NamedTemporaryFile("w", suffix=".extxyz", delete=True) as f:
        f.write(text)
        f.flush()
        structs = read_extxyz(f.name)
    # the extra per-atom columns
    lines = text.splitlines()
    i, k = 0, 0
    while i < len(lines) and k < len(structs):
        if not lines[i].strip():
            i += 1
            continue
        n = int(lines[i].split()[0])
        head = lines[i + 1]
        m = re.search(r"Properties=(\S+)", head)
        cols = m.group(1).split(":") if m else []
        spec = [(cols[j], cols[j + 1], int(cols[j + 2])) for j in range(0, len(cols), 3)]
        rows = [lines[i + 2 + a].split() for a in range(n)]
        c = 0
        for name, kind, width in spec:
            if name in ("move_mask", "tags"):
                vals = [r[c:c + width] for r in rows]
                if kind == "L":
                    structs[k][name] = np.array([v[0] in ("T", "True", "1") for v in vals])
                else:
                    structs[k][name] = np.array([int(v[0]) for v in vals])
            c += width
        i += 2 + n
        k += 1
    return structs


class OC20S2EF(DatasetBuilder):
    name = "oc20_s2ef_200k"
    description = "OC20 S2EF 200K training frames (adsorbates on catalyst slabs), energies and forces"

    def load(self, *, split: Optional[str], cache_dir: Path, energy: str = "adsorption",
             max_frames: Optional[int] = None, archive: Optional[str] = None, seed: int = 0, **_):
        if energy not in ("adsorption", "total"):
            raise ValueError("energy must be 'adsorption' or 'total'")
        path = Path(archive) if archive else fetch(OC20_200K[0], cache_dir / "oc20" / "s2ef_train_200K.tar",
                                                   OC20_200K[1])
        return select_split(seeded_splits(read_oc20_archive(path, energy, max_frames), seed), split)


# ----------------------------------------------------------------------------- Materials Project 2018
MP2018 = ("https://ndownloader.figshare.com/files/15087992", "4599ea88419c6a90bfb0dad2c2bf3733")


def parse_p1_cif(text: str) -> dict:
    """A P1 CIF (cell parameters and fractional sites, one symmetry operation) as a structure."""
    vals: Dict[str, float] = {}
    for key in ("_cell_length_a", "_cell_length_b", "_cell_length_c", "_cell_angle_alpha", "_cell_angle_beta",
                "_cell_angle_gamma"):
        m = re.search(re.escape(key) + r"\s+([-\d.eE+]+)", text)
        if m is None:
            raise ValueError(f"CIF without {key}")
        vals[key] = float(m.group(1))
    a, b, c = vals["_cell_length_a"], vals["_cell_length_b"], vals["_cell_length_c"]
    al, be, ga = (math.radians(vals[k]) for k in ("_cell_angle_alpha", "_cell_angle_beta", "_cell_angle_gamma"))
    cx = math.cos(be)
    cy = (math.cos(al) - math.cos(be) * math.cos(ga)) / math.sin(ga)
    cell = np.array([[a, 0.0, 0.0], [b * math.cos(ga), b * math.sin(ga), 0.0],
                     [c * cx, c * cy, c * math.sqrt(max(0.0, 1.0 - cx * cx - cy * cy))]])
    lines = text.splitlines()
    sites, header, in_loop = [], [], False
    for ln in lines:
        s = ln.strip()
        if s.startswith("loop_"):
            header, in_loop = [], True
            continue
        if in_loop and s.startswith("_"):
            header.append(s.split()[0])
            continue
        if in_loop and header and "_atom_site_fract_x" in header and s and not s.startswith(("_", "#", "loop_")):
            f = s.split()
            if len(f) < len(header):
                continue
            row = dict(zip(header, f))
            sym = row.get("_atom_site_type_symbol", row.get("_atom_site_label", ""))
            sym = re.match(r"[A-Z][a-z]?", sym).group(0)
            occ = float(row.get("_atom_site_occupancy", "1"))
            sites.append((sym, [float(row[f"_atom_site_fract_{x}"].split("(")[0]) for x in "xyz"], occ))
    if not sites:
        raise ValueError("CIF without atom sites")
    frac = np.array([p for _, p, _ in sites])
    return {"pos": torch.tensor(frac @ cell, dtype=torch.float64),
            "atomic_numbers": torch.tensor([ATOMIC_NUMBERS[s] for s, _, _ in sites]),
            "cell": torch.tensor(cell, dtype=torch.float64), "pbc": torch.ones(3, dtype=torch.bool)}


def read_mp2018(path, max_entries: Optional[int] = None) -> List[dict]:
    with zipfile.ZipFile(path) as z:
        name = next(n for n in z.namelist() if n.endswith(".json"))
        entries = json.loads(z.read(name).decode())
    out = []
    for e in entries[:max_entries] if max_entries else entries:
        s = parse_p1_cif(e["structure"])
        n = int(s["atomic_numbers"].shape[0])
        s["formation_energy_per_atom"] = float(e["formation_energy_per_atom"])
        s["energy"] = s["formation_energy_per_atom"] * n
        s["band_gap"] = float(e.get("band_gap", float("nan")))
        for key, label in (("K", "log10_bulk_modulus"), ("G", "log10_shear_modulus")):
            v = e.get(key)
            s[label] = float(v) if v is not None else float("nan")
        s["info"] = {"material_id": e.get("material_id")}
        out.append(s)
    return out


class MP2018(DatasetBuilder):
    name = "mp_2018"
    description = "Materials Project 2018.6.1 (MEGNet): formation energies, band gaps, elastic moduli"

    def load(self, *, split: Optional[str], cache_dir: Path, max_entries: Optional[int] = None,
             archive: Optional[str] = None, seed: int = 0, **_):
        path = Path(archive) if archive else fetch(MP2018[0], cache_dir / "mp" / "mp.2018.6.1.json.zip", MP2018[1])
        return select_split(seeded_splits(read_mp2018(path, max_entries), seed), split)


# ----------------------------------------------------------------------------- ASE SQLite databases
def _blob(value, dtype, shape=None):
    if value is None:
        return None
    a = np.frombuffer(value, dtype=dtype).copy()
    return a.reshape(shape) if shape is not None else a


def read_ase_db(path, selection: Optional[str] = None, limit: Optional[int] = None) -> List[dict]:
    """Rows of an ASE SQLite database (its ``systems`` table) as structure dicts."""
    con = sqlite3.connect(f"file:{Path(path)}?mode=ro", uri=True)
    try:
        cols = [r[1] for r in con.execute("PRAGMA table_info(systems)")]
        q = "SELECT * FROM systems" + (f" WHERE {selection}" if selection else "") + " ORDER BY id"
        if limit:
            q += f" LIMIT {int(limit)}"
        out = []
        for row in con.execute(q):
            r = dict(zip(cols, row))
            z = _blob(r["numbers"], np.int32)
            n = z.shape[0]
            s = {"pos": torch.tensor(_blob(r["positions"], np.float64, (n, 3))),
                 "atomic_numbers": torch.tensor(z.astype(np.int64))}
            cell = _blob(r.get("cell"), np.float64, (3, 3))
            pbc = int(r.get("pbc") or 0)
            if cell is not None and pbc:
                s["cell"] = torch.tensor(cell)
                s["pbc"] = torch.tensor([bool(pbc & 1), bool(pbc & 2), bool(pbc & 4)])
            if r.get("energy") is not None:
                s["energy"] = float(r["energy"])
            f = _blob(r.get("forces"), np.float64, (n, 3))
            if f is not None:
                s["forces"] = torch.tensor(f)
            st = _blob(r.get("stress"), np.float64)
            if st is not None:
                if st.shape[0] == 6:
                    xx, yy, zz, yz, xz, xy = st
                    st = np.array([[xx, xy, xz], [xy, yy, yz], [xz, yz, zz]])
                s["stress"] = torch.tensor(st.reshape(3, 3))
            q = _blob(r.get("initial_charges"), np.float64) if r.get("charges") is None else _blob(r["charges"],
                                                                                                   np.float64)
            if q is not None and q.shape[0] == n:
                s["charges"] = torch.tensor(q)
            kv = r.get("key_value_pairs")
            s["info"] = {"id": r.get("id"), **(json.loads(kv) if kv else {})}
            out.append(s)
        return out
    finally:
        con.close()


class AseDatabase(DatasetBuilder):
    name = "ase_db"
    description = "Any ASE SQLite database (path=...): positions, numbers, cell, energies, forces, stress"

    def load(self, *, split: Optional[str], cache_dir: Path, path: Optional[str] = None,
             selection: Optional[str] = None, limit: Optional[int] = None, seed: int = 0, **_):
        if path is None:
            raise ValueError("ase_db needs path=<database file>")
        items = read_ase_db(path, selection, limit)
        return items if split is None else select_split(seeded_splits(items, seed), split)


for _b in (OC20S2EF(), MP2018(), AseDatabase()):
    register_dataset(_b)
