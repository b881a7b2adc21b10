"""Reaction-energy training (GMTKN55-style): a reaction is a stoichiometric combination of species
energies, ``dE_r = sum_s nu_rs E_s``; its squared error against a reference (optionally Huber,
optionally scaled per reaction as in WTMAD-2) trains the model alongside the per-structure terms.

Records and conventions follow the reference (``src/xnn/common/train/reactions.py``): structures
``{"name", "subset"?, "pos", "atomic_numbers", ...}``, reactions ``{"species", "stoichiometry",
"reference", "subset"?, "weight"?, "scale"?}``, species looked up by ``(subset, name)`` then by name,
references in eV, kcal/mol or hartree.
"""
from __future__ import annotations

from typing import Iterator, Mapping, Optional, Sequence

import numpy as np
import torch
from torch import Tensor

from ..data import collate, structure_to_graph
from .losses import _sq

KCAL_MOL_TO_EV = 4.336410424180094e-2
HARTREE_TO_EV = 27.211386245988
UNITS = {"ev": 1.0, "kcal/mol": KCAL_MOL_TO_EV, "hartree": HARTREE_TO_EV}


def reaction_energies(species_energy: Tensor, stoichiometry: Tensor) -> Tensor:
    return stoichiometry.to(species_energy.dtype) @ species_energy


def reaction_energy_loss(species_energy: Tensor, stoichiometry: Tensor, reference: Tensor,
                         weight: Optional[Tensor] = None, scale: Optional[Tensor] = None,
                         huber_delta: float = 0.0) -> Tensor:
    """Weighted mean of the squared (or Huber) errors of the reaction energies."""
    err = reaction_energies(species_energy, stoichiometry) - reference.to(species_energy.dtype)
    if scale is not None:
        err = err * scale.to(err.dtype)
    sq = _sq(err, huber_delta)
    if weight is None:
        return sq.mean()
    w = weight.to(sq.dtype)
    return (w * sq).sum() / w.sum()


class ReactionSet:
    """Structures and the reactions over them."""

    def __init__(self, structures: Sequence[Mapping], reactions: Sequence[Mapping], units: str = "eV"):
        if units.lower() not in UNITS:
            raise ValueError(f"units must be one of 'eV', 'kcal/mol', 'hartree', got {units!r}")
        f = UNITS[units.lower()]
        self.structures = list(structures)
        where = {(s.get("subset"), s["name"]): k for k, s in enumerate(self.structures)}
        self.members, ref, wts, scl, self.labels = [], [], [], [], []
        for k, r in enumerate(reactions):
            sub = r.get("subset")
            try:
                idx = [where[(sub, nm)] if (sub, nm) in where else where[(None, nm)] for nm in r["species"]]
            except KeyError as exc:
                raise KeyError(f"reaction {k}: no structure for species {exc.args[0]!r}") from None
            if len(idx) != len(r["stoichiometry"]):
                raise ValueError(f"reaction {k}: {len(idx)} species but {len(r['stoichiometry'])} coefficients")
            self.members.append((idx, [float(c) for c in r["stoichiometry"]]))
            ref.append(f * float(r["reference"]))
            wts.append(float(r.get("weight", 1.0)))
            scl.append(float(r.get("scale", 1.0)))
            self.labels.append((sub, r.get("index", k)))
        self.reference = torch.tensor(ref, dtype=torch.float64)
        self.weight = torch.tensor(wts, dtype=torch.float64)
        self.scale = torch.tensor(scl, dtype=torch.float64)
        self._graphs: dict = {}

    @classmethod
    def from_gmtkn55(cls, data: Mapping, wtmad2: bool = False, scale: float = 56.84) -> "ReactionSet":
        """GMTKN55-style records (kcal/mol); ``wtmad2`` scales each reaction by ``scale / <|dE|>`` of
        its subset (the WTMAD-2 weighting)."""
        recs = [dict(r) for r in data["reactions"]]
        if wtmad2:
            sums: dict = {}
            for r in recs:
                n, s = sums.get(r["subset"], (0, 0.0))
                sums[r["subset"]] = (n + 1, s + abs(float(r["reference"])))
            for r in recs:
                n, s = sums[r["subset"]]
                r["scale"] = scale / (s / n)
        return cls(data["structures"], recs, units="kcal/mol")

    def __len__(self) -> int:
        return len(self.members)

    def subset(self, reactions: Sequence[int]) -> "ReactionSet":
        out = ReactionSet.__new__(ReactionSet)
        keep: dict = {}
        out.members = []
        for r in reactions:
            idx, coef = self.members[int(r)]
            out.members.append(([keep.setdefault(i, len(keep)) for i in idx], list(coef)))
        order = sorted(keep, key=keep.get)
        out.structures = [self.structures[i] for i in order]
        sel = torch.as_tensor([int(r) for r in reactions], dtype=torch.long)
        out.reference, out.weight, out.scale = self.reference[sel], self.weight[sel], self.scale[sel]
        out.labels = [self.labels[int(r)] for r in reactions]
        out._graphs = {k: [g[i] for i in order] for k, g in self._graphs.items()}
        return out

    def stoichiometry(self) -> Tensor:
        out = torch.zeros(len(self.members), len(self.structures), dtype=torch.float64)
        for r, (idx, coef) in enumerate(self.members):
            for i, c in zip(idx, coef):
                out[r, i] += c
        return out

    def graphs(self, cutoff: float) -> list:
        key = float(cutoff)
        if key not in self._graphs:
            self._graphs[key] = [structure_to_graph(dict(s), key) for s in self.structures]
        return self._graphs[key]

    def batches(self, size: int, shuffle: bool = True, seed: int = 0) -> Iterator["ReactionSet"]:
        order = np.random.default_rng(seed).permutation(len(self)) if shuffle else np.arange(len(self))
        for s in range(0, len(order), size):
            yield self.subset(order[s:s + size].tolist())

    def species_energies(self, model: torch.nn.Module, cutoff: float, batch_size: int = 32,
                         device: Optional[torch.device] = None) -> Tensor:
        gs, out = self.graphs(cutoff), []
        p = next(model.parameters(), None)
        for s in range(0, len(gs), batch_size):
            b = collate(gs[s:s + batch_size])
            if p is not None and b.pos.dtype != p.dtype:
                b.compute_dtype = p.dtype          # float64 geometry driving the model's dtype
            out.append(model(b.to(device) if device is not None else b)["energy"].reshape(-1))
        return torch.cat(out) if out else torch.zeros(0, dtype=torch.float64)

    def loss(self, species_energy: Tensor, huber_delta: float = 0.0) -> Tensor:
        dev = species_energy.device
        return reaction_energy_loss(species_energy, self.stoichiometry().to(dev), self.reference.to(dev),
                                    self.weight.to(dev), self.scale.to(dev), huber_delta)

    def errors(self, species_energy: Tensor) -> Tensor:
        dev = species_energy.device
        return reaction_energies(species_energy, self.stoichiometry().to(dev)) - self.reference.to(dev)
