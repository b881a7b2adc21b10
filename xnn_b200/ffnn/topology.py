"""Fixed molecular topology of the classical force fields: per-atom types, bonds and what follows
from them (angles, proper dihedrals, 1-2/1-3 exclusions, 1-4 and 1-5 pairs), impropers, and the
optional bond orders, structure-bound charges and residue positions.

Derivation rules, field names and the JSON file layout follow the reference
(``src/xnn/ffnn/models/topology.py:39-545``) so topologies and their files are interchangeable:
angles are unordered neighbour pairs of each centre, proper dihedrals are enumerated once per
bond, 1-4 pairs are dihedral ends not already 1-2/1-3, 1-5 pairs one bond beyond a dihedral.
"""
from __future__ import annotations

import itertools
import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import List, Optional, Sequence, Tuple, Union

import numpy as np

from ..data.elements import COVALENT_RADII


def guess_bonds(positions, atomic_numbers, cell=None, scale: float = 1.2) -> List[Tuple[int, int]]:
    """Bonds ``(i, j)``, ``i < j``, of atoms closer than ``scale`` times the sum of their covalent
    radii (minimum over periodic images when ``cell`` is given)."""
    pos = np.asarray(positions, dtype=float)
    z = np.asarray(atomic_numbers, dtype=int)
    radii = np.array([COVALENT_RADII[int(v)] for v in z])
    n = len(z)
    if n < 2:
        return []
    if cell is not None:
        cell = np.asarray(cell, dtype=float)
        inv = np.linalg.inv(cell)
        normals = np.cross(np.roll(cell, -1, 0), np.roll(cell, -2, 0))
        spacing = abs(np.linalg.det(cell)) / np.linalg.norm(normals, axis=1)
        reach = scale * 2.0 * radii.max() / spacing
        reps = np.maximum(1, np.floor(reach + 0.5).astype(int))
        offsets = np.array(list(itertools.product(*[range(-r, r + 1) for r in reps])), dtype=float)
    bonds = []
    step = max(1, int(2e6 // n))
    for a in range(0, n - 1, step):
        b = min(n - 1, a + step)
        vec = pos[None, :, :] - pos[a:b, None, :]
        lim = scale * (radii[a:b, None] + radii[None, :])
        upper = np.arange(n)[None, :] > np.arange(a, b)[:, None]
        if cell is None:
            rows, cols = np.nonzero((np.sqrt((vec * vec).sum(-1)) < lim) & upper)
        else:
            frac = vec @ inv
            frac -= np.round(frac)
            rows, cols = np.nonzero(((np.abs(frac) < reach) | (reach > 0.5)).all(-1) & upper)
            cand = (frac[rows, cols][:, None, :] + offsets) @ cell
            keep = np.sqrt((cand * cand).sum(-1)).min(-1) < lim[rows, cols]
            rows, cols = rows[keep], cols[keep]
        bonds.extend(zip((rows + a).tolist(), cols.tolist()))
    return sorted(bonds)


@dataclass
class MolecularTopology:
    types: List[str]
    bonds: List[Tuple[int, int]]
    bond_orders: List[float] = field(default_factory=list)
    angles: List[Tuple[int, int, int]] = field(default_factory=list)
    dihedrals: List[Tuple[int, int, int, int]] = field(default_factory=list)
    impropers: List[Tuple[int, int, int, int]] = field(default_factory=list)
    improper_keys: List[str] = field(default_factory=list)
    exclusions: List[Tuple[int, int]] = field(default_factory=list)
    pairs14: List[Tuple[int, int]] = field(default_factory=list)
    pairs15: List[Tuple[int, int]] = field(default_factory=list)
    charges: List[float] = field(default_factory=list)
    residues: list = field(default_factory=list)
    residue_names: list = field(default_factory=list)

    @property
    def n_atoms(self) -> int:
        return len(self.types)

    @classmethod
    def from_bonds(cls, types: Sequence[str], bonds: Sequence[Sequence[int]], impropers: Sequence = (),
                   improper_keys: Sequence[str] = (), bond_orders: Optional[Sequence[float]] = None,
                   charges: Optional[Sequence[float]] = None, residues: Optional[Sequence] = None,
                   residue_names: Optional[Sequence[str]] = None) -> "MolecularTopology":
        n = len(types)
        if bond_orders is not None and len(bond_orders) != len(bonds):
            raise ValueError(f"got {len(bond_orders)} bond orders for {len(bonds)} bonds")
        if charges is not None and len(charges) != n:
            raise ValueError(f"got {len(charges)} charges for {n} atoms")
        if residues is not None and len(residues) != n:
            raise ValueError(f"got {len(residues)} residue entries for {n} atoms")
        if improper_keys and len(impropers) != len(improper_keys):
            raise ValueError(f"impropers and improper_keys must have the same length (got {len(impropers)} and "
                             f"{len(improper_keys)}); leave improper_keys empty to resolve impropers by atom class")
        order, seen = {}, set()
        for m, pair in enumerate(bonds):
            i, j = int(pair[0]), int(pair[1])
            if not (0 <= i < n and 0 <= j < n):
                raise ValueError(f"bond ({i}, {j}) is out of range for {n} atoms")
            if i == j:
                raise ValueError(f"bond ({i}, {j}) joins an atom to itself")
            key = (min(i, j), max(i, j))
            if key in seen:
                raise ValueError(f"duplicate bond {key}")
            seen.add(key)
            if bond_orders is not None:
                order[key] = float(bond_orders[m])
        blist = sorted(seen)
        nbr = [[] for _ in range(n)]
        for i, j in blist:
            nbr[i].append(j)
            nbr[j].append(i)
        for x in nbr:
            x.sort()
        angles = [(x[a], j, x[b]) for j, x in enumerate(nbr) for a in range(len(x)) for b in range(a + 1, len(x))]
        dihedrals, done = [], set()
        for j, k in blist:
            for i in nbr[j]:
                if i == k:
                    continue
                for l in nbr[k]:
                    if l in (i, j):
                        continue
                    quad = (i, j, k, l)
                    canon = min(quad, quad[::-1])
                    if canon not in done:
                        done.add(canon)
                        dihedrals.append(quad)
        excl = set(blist) | {(min(i, k), max(i, k)) for i, _, k in angles}
        p14 = {(min(i, l), max(i, l)) for i, _, _, l in dihedrals} - excl
        p15 = set()
        for i, j, k, l in dihedrals:
            for m in nbr[l]:
                if m not in (i, j, k):
                    p15.add((min(i, m), max(i, m)))
            for m in nbr[i]:
                if m not in (j, k, l):
                    p15.add((min(m, l), max(m, l)))
        p15 -= excl | p14
        return cls(types=list(types), bonds=blist, bond_orders=[order[b] for b in blist] if bond_orders is not None
                   else [], angles=angles, dihedrals=dihedrals, impropers=[tuple(int(x) for x in im) for im in impropers],
                   improper_keys=list(improper_keys), exclusions=sorted(excl), pairs14=sorted(p14),
                   pairs15=sorted(p15), charges=[float(q) for q in charges] if charges is not None else [],
                   residues=[None if r is None else (int(r[0]), int(r[1])) for r in residues]
                   if residues is not None else [],
                   residue_names=[str(x) for x in residue_names] if residue_names is not None else [])

    @classmethod
    def from_structure(cls, positions, atomic_numbers, types: Sequence[str], bonds=None, cell=None,
                       scale: float = 1.2, **kw) -> "MolecularTopology":
        """A topology with explicit types and bonds guessed from the coordinates when not given."""
        if len(types) != len(atomic_numbers):
            raise ValueError(f"got {len(types)} types for {len(atomic_numbers)} atoms")
        if bonds is None:
            bonds = guess_bonds(positions, atomic_numbers, cell=cell, scale=scale)
        return cls.from_bonds(types, bonds, **kw)

    def replicate(self, n_copies: int) -> "MolecularTopology":
        """``n_copies`` consecutive molecules (atom ``a`` of copy ``c`` is ``c * n_atoms + a``)."""
        n = self.n_atoms
        n_res = 1 + max((r[0] for r in self.residues if r is not None), default=-1)

        def sh(items, off):
            return [tuple(x + off for x in it) for it in items]
        out = MolecularTopology(types=list(self.types) * n_copies, bonds=[], charges=list(self.charges) * n_copies,
                                residue_names=list(self.residue_names) * n_copies)
        for c in range(n_copies):
            off = c * n
            out.residues += [None if r is None else (r[0] + c * n_res, r[1]) for r in self.residues]
            out.bonds += sh(self.bonds, off)
            out.bond_orders += list(self.bond_orders)
            out.angles += sh(self.angles, off)
            out.dihedrals += sh(self.dihedrals, off)
            out.impropers += sh(self.impropers, off)
            out.improper_keys += list(self.improper_keys)
            out.exclusions += sh(self.exclusions, off)
            out.pairs14 += sh(self.pairs14, off)
            out.pairs15 += sh(self.pairs15, off)
        return out

    def save(self, path: Union[str, Path]) -> None:
        """JSON with the independent data (types, bonds, impropers and the optional lists)."""
        data = {"types": self.types, "bonds": [list(b) for b in self.bonds],
                "impropers": [list(im) for im in self.impropers], "improper_keys": self.improper_keys}
        if self.bond_orders:
            data["bond_orders"] = list(self.bond_orders)
        if self.charges:
            data["charges"] = list(self.charges)
        if self.residues:
            data["residues"] = [None if r is None else list(r) for r in self.residues]
        if self.residue_names:
            data["residue_names"] = list(self.residue_names)
        Path(path).write_text(json.dumps(data, indent=2) + "\n")


def read_topology(path: Union[str, Path]) -> MolecularTopology:
    d = json.loads(Path(path).read_text())
    return MolecularTopology.from_bonds(d["types"], d["bonds"], impropers=d.get("impropers", ()),
                                        improper_keys=d.get("improper_keys", ()), bond_orders=d.get("bond_orders"),
                                        charges=d.get("charges"), residues=d.get("residues"),
                                        residue_names=d.get("residue_names"))
