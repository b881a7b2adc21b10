"""Reaction-energy training (GMTKN55-style benchmarks).

A reaction ``r`` combines species energies with stoichiometric coefficients,
``dE_r = sum_s nu_rs E_s``. Its error against a reference value (optionally Huber-clipped and
optionally multiplied by a per-reaction factor, which is how the WTMAD-2 weighting enters) is a
loss term trained next to the per-structure energy and force terms.

Storage: the coefficients are kept as coordinate triples ``(reaction, species, nu)`` rather than
a dense reaction x species matrix, so a batch of reactions evaluates with one ``index_add`` over
its terms and drawing a batch only renumbers the species that batch touches. The dense matrix
is still available (:meth:`ReactionSet.stoichiometry`) for callers that want it.

Record formats are the reference's (``src/xnn/common/train/reactions.py``): structures are
dictionaries ``{"name", "subset"?, "pos", "atomic_numbers", ...}``; reactions are
``{"species", "stoichiometry", "reference", "subset"?, "weight"?, "scale"?, "index"?}``; a
species name is looked up inside the reaction's subset first and then without a subset;
references are in eV, kcal/mol or hartree.
"""
from __future__ import annotations

from typing import Dict, Iterator, List, Mapping, Optional, Sequence, Tuple

import numpy as np
import torch
from torch import Tensor

from ..data import collate, structure_to_graph
from .losses import _sq

KCAL_MOL_TO_EV = 4.336410424180094e-2
HARTREE_TO_EV = 27.211386245988
UNITS = {"ev": 1.0, "kcal/mol": KCAL_MOL_TO_EV, "hartree": HARTREE_TO_EV}


def reaction_energies(species_energy: Tensor, stoichiometry: Tensor) -> Tensor:
    """``dE = nu @ E`` for a dense ``(reactions, species)`` coefficient matrix."""
    return torch.mv(stoichiometry.to(species_energy.dtype), species_energy)


def _reduce(err: Tensor, weight: Optional[Tensor], scale: Optional[Tensor], huber_delta: float) -> Tensor:
    if scale is not None:
        err = err * scale.to(err.dtype)
    per = _sq(err, huber_delta)
    if weight is None:
        return per.mean()
    w = weight.to(per.dtype)
    return torch.dot(w, per) / w.sum()


def reaction_energy_loss(species_energy: Tensor, stoichiometry: Tensor, reference: Tensor,
                         weight: Optional[Tensor] = None, scale: Optional[Tensor] = None,
                         huber_delta: float = 0.0) -> Tensor:
    """Weighted mean of the squared (or Huber) errors of the reaction energies."""
    err = reaction_energies(species_energy, stoichiometry) - reference.to(species_energy.dtype)
    return _reduce(err, weight, scale, huber_delta)


class ReactionSet:
    """Structures and the reactions defined over them."""

    def __init__(self, structures: Sequence[Mapping], reactions: Sequence[Mapping], units: str = "eV"):
        factor = UNITS.get(units.lower())
        if factor is None:
            raise ValueError(f"units must be one of 'eV', 'kcal/mol', 'hartree', got {units!r}")
        self.structures = list(structures)
        lookup: Dict[Tuple[Optional[str], str], int] = {}
        for k, s in enumerate(self.structures):
            lookup.setdefault((s.get("subset"), s["name"]), k)
        rows: List[int] = []
        cols: List[int] = []
        nus: List[float] = []
        values = np.zeros((len(reactions), 3))          # reference (eV), weight, scale
        self.labels = []
        for k, rec in enumerate(reactions):
            names, coefs = list(rec["species"]), list(rec["stoichiometry"])
            if len(names) != len(coefs):
                raise ValueError(f"reaction {k}: {len(names)} species but {len(coefs)} coefficients")
            sub = rec.get("subset")
            for name, nu in zip(names, coefs):
                s = lookup.get((sub, name), lookup.get((None, name)))
                if s is None:
                    raise KeyError(f"reaction {k}: no structure for species {name!r}")
                rows.append(k)
                cols.append(s)
                nus.append(float(nu))
            values[k] = (factor * float(rec["reference"]), float(rec.get("weight", 1.0)),
                         float(rec.get("scale", 1.0)))
            self.labels.append((sub, rec.get("index", k)))
        self._set_terms(torch.tensor(rows, dtype=torch.long), torch.tensor(cols, dtype=torch.long),
                        torch.tensor(nus, dtype=torch.float64))
        v = torch.from_numpy(values)
        self.reference, self.weight, self.scale = v[:, 0].clone(), v[:, 1].clone(), v[:, 2].clone()
        self._graphs: Dict[float, list] = {}

    def _set_terms(self, rows: Tensor, cols: Tensor, nu: Tensor) -> None:
        self.term_reaction, self.term_species, self.term_nu = rows, cols, nu

    @classmethod
    def from_gmtkn55(cls, data: Mapping, wtmad2: bool = False, scale: float = 56.84) -> "ReactionSet":
        """GMTKN55-style records (kcal/mol). With ``wtmad2`` every reaction is multiplied by
        ``scale / mean |dE_ref|`` of its subset, the WTMAD-2 weighting."""
        recs = [dict(r) for r in data["reactions"]]
        if wtmad2:
            by_subset: Dict[str, List[float]] = {}
            for r in recs:
                by_subset.setdefault(r["subset"], []).append(abs(float(r["reference"])))
            mean_abs = {k: float(np.mean(v)) for k, v in by_subset.items()}
            for r in recs:
                r["scale"] = scale / mean_abs[r["subset"]]
        return cls(data["structures"], recs, units="kcal/mol")

    def __len__(self) -> int:
        return int(self.reference.shape[0])

    def subset(self, reactions: Sequence[int]) -> "ReactionSet":
        """The given reactions over only the species they use (numbered by first use)."""
        sel = torch.as_tensor([int(r) for r in reactions], dtype=torch.long)
        # terms of the selected reactions, in selection order, keeping each reaction's term order
        pos_of = torch.full((len(self),), -1, dtype=torch.long)
        pos_of[sel] = torch.arange(sel.numel())
        new_row = pos_of[self.term_reaction]
        keep = new_row >= 0
        order = torch.argsort(new_row[keep] * (self.term_reaction.numel() + 1)
                              + torch.arange(self.term_reaction.numel())[keep])
        rows, cols, nu = new_row[keep][order], self.term_species[keep][order], self.term_nu[keep][order]
        used, first = np.unique(cols.numpy(), return_index=True)
        by_first = used[np.argsort(first)]                  # species in order of first use
        renum = torch.full((len(self.structures),), -1, dtype=torch.long)
        renum[torch.from_numpy(by_first)] = torch.arange(len(by_first))
        out = ReactionSet.__new__(ReactionSet)
        out.structures = [self.structures[i] for i in by_first.tolist()]
        out._set_terms(rows, renum[cols], nu)
        out.reference, out.weight, out.scale = self.reference[sel], self.weight[sel], self.scale[sel]
        out.labels = [self.labels[i] for i in sel.tolist()]
        out._graphs = {k: [g[i] for i in by_first.tolist()] for k, g in self._graphs.items()}
        return out

    def stoichiometry(self) -> Tensor:
        """Dense ``(reactions, species)`` coefficients (repeated species add up)."""
        out = torch.zeros(len(self), len(self.structures), dtype=torch.float64)
        return out.index_put_((self.term_reaction, self.term_species), self.term_nu, accumulate=True)

    def graphs(self, cutoff: float) -> list:
        key = float(cutoff)
        if key not in self._graphs:
            self._graphs[key] = [structure_to_graph(dict(s), key) for s in self.structures]
        return self._graphs[key]

    def batches(self, size: int, shuffle: bool = True, seed: int = 0) -> Iterator["ReactionSet"]:
        idx = np.arange(len(self))
        if shuffle:
            idx = np.random.default_rng(seed).permutation(idx)
        for start in range(0, len(idx), size):
            yield self.subset(idx[start:start + size].tolist())

    def species_energies(self, model: torch.nn.Module, cutoff: float, batch_size: int = 32,
                         device: Optional[torch.device] = None) -> Tensor:
        """Model energy of every structure of the set, in order."""
        gs = self.graphs(cutoff)
        if not gs:
            return torch.zeros(0, dtype=torch.float64)
        p = next(model.parameters(), None)
        parts = []
        for s in range(0, len(gs), batch_size):
            b = collate(gs[s:s + batch_size])
            if p is not None and b.pos.dtype != p.dtype:
                b.compute_dtype = p.dtype          # float64 geometry driving the model's dtype
            if device is not None:
                b = b.to(device)
            parts.append(model(b)["energy"].reshape(-1))
        return torch.cat(parts)

    def errors(self, species_energy: Tensor) -> Tensor:
        """``dE_model - dE_ref`` per reaction, by summing the coefficient terms."""
        dev, dt = species_energy.device, species_energy.dtype
        terms = self.term_nu.to(dev, dt) * species_energy.index_select(0, self.term_species.to(dev))
        dE = torch.zeros(len(self), dtype=dt, device=dev).index_add_(0, self.term_reaction.to(dev), terms)
        return dE - self.reference.to(dev, dt)

    def loss(self, species_energy: Tensor, huber_delta: float = 0.0) -> Tensor:
        dev = species_energy.device
        return _reduce(self.errors(species_energy), self.weight.to(dev), self.scale.to(dev), huber_delta)
