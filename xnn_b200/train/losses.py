"""Weighted training loss (``src/xnn/common/train/losses.py:277``).

Terms (each skipped when its weight is zero or its label absent):

* energy: per-atom energy error ``(E - E_ref) / n_atoms``, squared, averaged over structures;
* forces: squared component error averaged over atoms and components, with per-atom
  weights ``u_i = weight * force_weight * atom_force_weight``;
* stress, dipole, polarizability, charges, properties: mean squared errors.

Per-structure ``weight`` and per-term weights make every mean a weighted mean; label
masks restrict a term to the labelled structures; ``huber_delta > 0`` replaces the
square by a Huber function. No host synchronisation happens here, so the loss can be
captured in a CUDA graph; the logged values are tensors.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
from torch import Tensor

from ..data import AtomicGraph


def _sq(r: Tensor, delta: float) -> Tensor:
    if delta and delta > 0:
        a = r.abs()
        return torch.where(a <= delta, r * r, 2.0 * delta * a - delta * delta)
    return r * r


def _wmean(values: Tensor, w: Optional[Tensor]) -> Tuple[Tensor, Tensor]:
    if w is None:
        return values.mean(), torch.tensor(float(values.numel()), device=values.device)
    w = w.to(values.dtype)
    den = w.sum()
    return (values * w).sum() / den.clamp_min(1e-12), den


def weighted_loss(pred: Dict[str, Tensor], data: AtomicGraph, energy_weight: float,
                  force_weight: float, stress_weight: float = 0.0, *, dipole_weight: float = 0.0,
                  polarizability_weight: float = 0.0, charge_weight: float = 0.0,
                  property_weight: float = 0.0, huber_delta: float = 0.0,
                  huber_delta_energy: Optional[float] = None,
                  huber_delta_forces: Optional[float] = None,
                  huber_delta_stress: Optional[float] = None,
                  counts: Optional[dict] = None, parts: Optional[dict] = None) -> Tuple[Tensor, Dict[str, Tensor]]:
    """Weighted sum of the loss terms; ``parts``, when given, receives every weighted term under
    its :data:`LOSS_TERMS` name (the input of :class:`UncertaintyWeights`)."""
    logs: Dict[str, Tensor] = {}
    total = None
    dev = data.pos.device

    def add(term: Tensor, w: float, key: str, den: Tensor):
        nonlocal total
        logs[key] = term.detach()
        if counts is not None:
            counts[key] = (den.detach(), w)
        if parts is not None:
            parts[_PART_NAME[key]] = term * w
        total = term * w if total is None else total + term * w

    sw = data.weight

    def struct_w(mask: Optional[Tensor], extra: Optional[Tensor]) -> Optional[Tensor]:
        w = sw
        if extra is not None:
            w = extra if w is None else w * extra
        if mask is not None:
            m = mask.to(torch.float64)
            w = m if w is None else w * m
        return w

    if energy_weight > 0 and data.energy is not None and "energy" in pred:
        n = data.n_atoms.to(torch.float64)
        r = (pred["energy"].to(torch.float64) - data.energy.to(torch.float64)) / n
        d = huber_delta if huber_delta_energy is None else huber_delta_energy
        term, den = _wmean(_sq(r, d), struct_w(data.energy_mask, data.energy_weight))
        add(term, energy_weight, "energy", den)
    if force_weight > 0 and data.forces is not None and "forces" in pred:
        r = pred["forces"] - data.forces.to(pred["forces"].dtype)
        d = huber_delta if huber_delta_forces is None else huber_delta_forces
        sq = _sq(r, d).sum(-1) / 3.0
        w = struct_w(data.forces_mask, data.force_weight)
        wa = None if w is None else w.index_select(0, data.batch)
        if data.atom_force_weight is not None:
            wa = data.atom_force_weight if wa is None else wa * data.atom_force_weight
        term, den = _wmean(sq, wa)
        add(term, force_weight, "forces", den)
    if stress_weight > 0 and data.stress is not None and "stress" in pred:
        r = pred["stress"] - data.stress.to(pred["stress"].dtype)
        d = huber_delta if huber_delta_stress is None else huber_delta_stress
        sq = _sq(r, d).reshape(r.shape[0], -1).mean(-1)
        term, den = _wmean(sq, struct_w(data.stress_mask, data.stress_weight))
        add(term, stress_weight, "stress", den)
    if dipole_weight > 0 and data.dipole is not None and "dipole" in pred:
        sq = _sq(pred["dipole"] - data.dipole, huber_delta).mean(-1)
        term, den = _wmean(sq, struct_w(data.dipole_mask, None))
        add(term, dipole_weight, "dipole", den)
    if polarizability_weight > 0 and data.polarizability is not None and "polarizability" in pred:
        sq = _sq(pred["polarizability"] - data.polarizability, huber_delta).reshape(-1, 9).mean(-1)
        term, den = _wmean(sq, struct_w(data.polarizability_mask, None))
        add(term, polarizability_weight, "polarizability", den)
    if charge_weight > 0 and data.charges is not None and "charges" in pred:
        sq = _sq(pred["charges"] - data.charges, huber_delta)
        w = struct_w(data.charges_mask, None)
        term, den = _wmean(sq, None if w is None else w.index_select(0, data.batch))
        add(term, charge_weight, "charges", den)
    if property_weight > 0 and data.properties is not None and "properties" in pred:
        sq = _sq(pred["properties"] - data.properties, huber_delta).reshape(data.num_graphs, -1).mean(-1)
        term, den = _wmean(sq, struct_w(data.properties_mask, None))
        add(term, property_weight, "properties", den)
    if total is None:
        total = torch.zeros((), device=dev, dtype=torch.float64)
    return total, logs


#: the weighted loss terms by name, with the config weight that switches each on
LOSS_TERMS = {"energy_mse": "energy_weight", "force_mse": "force_weight", "stress_mse": "stress_weight",
              "dipole_mse": "dipole_weight", "polarizability_mse": "polarizability_weight",
              "charge_mse": "charge_weight", "property_mse": "property_weight"}
_PART_NAME = {"energy": "energy_mse", "forces": "force_mse", "stress": "stress_mse", "dipole": "dipole_mse",
              "polarizability": "polarizability_mse", "charges": "charge_mse", "properties": "property_mse"}


class UncertaintyWeights(torch.nn.Module):
    """Learned balance of the loss terms (Kendall, Gal & Cipolla, CVPR 2018, homoscedastic task
    uncertainty): term ``L_k`` (already times its config weight) contributes
    ``exp(-2 s_k) L_k / 2 + s_k`` with a trainable ``s_k = log sigma_k`` starting at 0; a term
    without an ``s_k`` adds unchanged. Parity: ``src/xnn/common/train/losses.py:529-585``
    (``optim.loss_weighting: uncertainty``)."""

    def __init__(self, names):
        super().__init__()
        self.log_sigma = torch.nn.ParameterDict({n: torch.nn.Parameter(torch.zeros(())) for n in names})

    def forward(self, parts: Dict[str, Tensor]) -> Tensor:
        out = None
        for name, term in parts.items():
            if name in self.log_sigma:
                ls = self.log_sigma[name].to(term.dtype)
                term = 0.5 * torch.exp(-2.0 * ls) * term + ls
            out = term if out is None else out + term
        if out is None:
            return next(iter(self.log_sigma.values())).new_zeros(())
        return out

    def sigmas(self) -> Dict[str, float]:
        return {n: float(torch.exp(p.detach())) for n, p in self.log_sigma.items()}


def error_metrics(pred: Dict[str, Tensor], data: AtomicGraph) -> Dict[str, Tensor]:
    """Sums of absolute and squared errors with their counts (pooled over batches by the caller)."""
    out: Dict[str, Tensor] = {}
    if data.energy is not None and "energy" in pred:
        r = (pred["energy"].detach().to(torch.float64) - data.energy) / data.n_atoms
        m = data.energy_mask
        if m is not None:
            r = r[m]
        out["energy_abs"], out["energy_sq"] = r.abs().sum(), (r * r).sum()
        out["energy_n"] = torch.tensor(float(r.numel()), device=r.device)
    if data.forces is not None and "forces" in pred:
        r = (pred["forces"].detach() - data.forces).to(torch.float64)
        w = data.atom_force_weight
        if w is not None:
            r = r * (w > 0)[:, None]
            n = (w > 0).sum() * 3.0
        else:
            n = torch.tensor(float(r.numel()), device=r.device)
        out["forces_abs"], out["forces_sq"], out["forces_n"] = r.abs().sum(), (r * r).sum(), n
    if data.stress is not None and "stress" in pred:
        r = (pred["stress"].detach() - data.stress).to(torch.float64)
        out["stress_abs"], out["stress_sq"] = r.abs().sum(), (r * r).sum()
        out["stress_n"] = torch.tensor(float(r.numel()), device=r.device)
    return out
