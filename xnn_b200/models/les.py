"""Latent Ewald Summation (LES): a long-range energy for any model with invariant node features.

Behaviour follows the reference's ``src/xnn/common/models/les.py`` (``EwaldSummation`` at
``:138``, ``LatentEwald`` at ``:600``), itself after Cheng, npj Comput Mater 11, 80 (2025): a
small MLP maps each atom's invariant features to latent charges ``q`` (``n_channels`` per atom)
and the Ewald energy of those charges is added to the short-range energy,

    E_lr = (2 / V) sum_{k in half space, 0 < |k| <= 2 pi / dl} f(k) |S(k)|^2,
    S(k) = sum_i q_i exp(i k . r_i),   f(k) = exp(-sigma^2 k^2 / 2) / k^2   (exponent 1)

for periodic structures, with the 1/r^6 kernel of the paper's eq 5 for ``exponent=6``; and the
Gaussian-screened direct sum ``sum_{i != j} q_i q_j erf(r / (sqrt 2 sigma)) / (4 pi r)`` plus the
self term for molecules. The conventions that fix the numbers are kept: the half-space
enumeration of the wave vectors (leading nonzero index positive, weight 2), the ``1e-9``
relative slack on the cutoff shell, the ``1e-6`` offset in the real-space denominator and the
``1 / (4 pi)`` normalisation, so energies of the two implementations agree to rounding.

Not built: the charge-equilibration solve and fragment constraints of the reference
(``charge_solve``, ``fragments``) and its particle-mesh variant of this sum (``method="pme"``).
"""
from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch
from torch import Tensor, nn

from ..data import elements
from ..data.atomic_graph import AtomicGraph
from ..ops.scatter import cell_volume, scatter_sum
from .base import InteratomicPotential

#: Coulomb constant e^2 / (4 pi eps0) in eV Angstrom
COULOMB_EV_A = 14.399645478425668
#: latent charge of one elementary charge: two latent charges interact as q1 q2 / (2 pi r)
LATENT_CHARGE_PER_E = math.sqrt(2.0 * math.pi * COULOMB_EV_A)


def intra_structure_pairs(batch: Tensor, num_graphs: int) -> Tuple[Tensor, Tensor]:
    """All ordered pairs ``(i, j)``, ``i != j``, of atoms of the same structure."""
    order = torch.argsort(batch, stable=True)
    counts = torch.bincount(batch, minlength=num_graphs)
    start = torch.cumsum(counts, 0) - counts
    graph = batch[order]
    per_atom = counts[graph]
    i = torch.repeat_interleave(torch.arange(batch.numel(), device=batch.device), per_atom)
    first = torch.cumsum(per_atom, 0) - per_atom
    local = torch.arange(i.numel(), device=batch.device) - torch.repeat_interleave(first, per_atom)
    j = start[graph[i]] + local
    keep = i != j
    return order[i[keep]], order[j[keep]]


def periodic_structures(cell: Optional[Tensor], pbc: Optional[Tensor], num_graphs: int,
                        device: torch.device) -> Tensor:
    if cell is None:
        return torch.zeros(num_graphs, dtype=torch.bool, device=device)
    periodic = cell.abs().sum(dim=(-2, -1)) > 1e-6
    if pbc is not None:
        periodic = periodic & pbc.any(-1)
    return periodic


class EwaldSummation(nn.Module):
    """Ewald energy of a per-atom latent variable ``q`` (see module notes)."""

    def __init__(self, dl: float = 2.0, sigma: float = 1.0, exponent: int = 1,
                 remove_self_interaction: bool = False, atom_block: int = 4096):
        super().__init__()
        if exponent not in (1, 6):
            raise ValueError(f"exponent must be 1 or 6, got {exponent}")
        self.dl, self.sigma, self.exponent = float(dl), float(sigma), int(exponent)
        self.remove_self_interaction = bool(remove_self_interaction)
        self.atom_block = int(atom_block)

    def kernel(self, k2: Tensor) -> Tensor:
        """``f(k)`` of the reciprocal sum for squared wave numbers ``k2``."""
        hs = 0.5 * self.sigma ** 2
        if self.exponent == 1:
            return torch.exp(-hs * k2) / k2
        u2 = hs * k2
        u = torch.sqrt(u2)
        tail = math.sqrt(math.pi) * torch.special.erfc(u) + (0.5 / u ** 3 - 1.0 / u) * torch.exp(-u2)
        return -(k2 ** 1.5 * tail)

    def self_energy(self, q: Tensor) -> Tensor:
        return q.square().sum() / (self.sigma * (2.0 * math.pi) ** 1.5)

    def wave_vectors(self, cell: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
        """Integer triples of one half space inside ``|k| <= 2 pi / dl``, their wave vectors and
        squared lengths, for a row-vector ``cell (3, 3)``."""
        device, dtype = cell.device, cell.dtype
        recip = 2.0 * math.pi * torch.linalg.inv(cell).T
        lengths = torch.linalg.norm(cell, dim=1).tolist()
        na, nb, nc = (max(int(float(L) / self.dl + 1e-9), 1) for L in lengths)
        ar = lambda lo, hi: torch.arange(lo, hi + 1, device=device)   # noqa: E731
        zero = torch.zeros(1, dtype=torch.long, device=device)
        grid = torch.cat([torch.cartesian_prod(ar(1, na), ar(-nb, nb), ar(-nc, nc)),
                          torch.cartesian_prod(zero, ar(1, nb), ar(-nc, nc)),
                          torch.cartesian_prod(zero, zero, ar(1, nc))])
        kpts = grid.to(dtype) @ recip
        k2 = kpts.square().sum(1)
        kc2 = (2.0 * math.pi / self.dl) ** 2
        keep = (k2 > kc2 * 1e-12) & (k2 <= kc2 * (1.0 + 1e-9))
        return grid[keep], kpts[keep], k2[keep]

    def reciprocal(self, pos: Tensor, q: Tensor, cell: Tensor) -> Tensor:
        """Reciprocal-space energy of one periodic structure (scalar), atoms in blocks."""
        _, kpts, k2 = self.wave_vectors(cell)
        re = im = None
        for a0 in range(0, pos.shape[0], self.atom_block):
            ang = pos[a0:a0 + self.atom_block] @ kpts.T                     # (n_b, M)
            qb = q[a0:a0 + self.atom_block]
            r_, i_ = torch.cos(ang).T @ qb, torch.sin(ang).T @ qb            # (M, C)
            re = r_ if re is None else re + r_
            im = i_ if im is None else im + i_
        energy = 2.0 * (self.kernel(k2)[:, None] * (re.square() + im.square())).sum() / cell_volume(cell)
        if self.remove_self_interaction and self.exponent == 1:
            energy = energy - self.self_energy(q)
        return energy

    def realspace_single(self, pos: Tensor, q: Tensor) -> Tensor:
        if self.exponent != 1:
            raise ValueError("the real-space sum supports exponent=1 only")
        diag = torch.eye(pos.shape[0], dtype=torch.bool, device=pos.device)
        d2 = (pos[:, None, :] - pos[None, :, :]).square().sum(-1)
        dist = d2.masked_fill(diag, 1.0).sqrt()
        kern = torch.special.erf(dist / (self.sigma * math.sqrt(2.0))) / (dist + 1e-6)
        kern = kern.masked_fill(diag, 0.0)
        energy = (q * (kern @ q)).sum() / (4.0 * math.pi)
        if not self.remove_self_interaction:
            energy = energy + self.self_energy(q)
        return energy

    def realspace_batch(self, pos: Tensor, q: Tensor, batch: Tensor, num_graphs: int) -> Tensor:
        if self.exponent != 1:
            raise ValueError("the real-space sum supports exponent=1 only")
        i, j = intra_structure_pairs(batch, num_graphs)
        dist = torch.linalg.norm(pos[i] - pos[j], dim=-1)
        pair = (q[i] * q[j]).sum(-1) * torch.special.erf(dist / (self.sigma * math.sqrt(2.0))) / (dist + 1e-6)
        energy = scatter_sum(pair, batch[i], num_graphs) / (4.0 * math.pi)
        if not self.remove_self_interaction:
            norm = self.sigma * (2.0 * math.pi) ** 1.5
            energy = energy + scatter_sum(q.square().sum(-1), batch, num_graphs) / norm
        return energy

    def forward(self, q: Tensor, pos: Tensor, batch: Tensor, num_graphs: int, cell: Optional[Tensor],
                pbc: Optional[Tensor] = None) -> Tensor:
        """Long-range energy per structure ``(B,)``."""
        if q.dim() == 1:
            q = q[:, None]
        if cell is None:
            if num_graphs == 1:
                return self.realspace_single(pos, q).reshape(1)
            return self.realspace_batch(pos, q, batch, num_graphs)
        periodic = periodic_structures(cell, pbc, num_graphs, pos.device)
        if num_graphs == 1 and not bool(periodic[0]):
            return self.realspace_single(pos, q).reshape(1)
        molecular = ~periodic[batch]
        out = self.realspace_batch(pos[molecular], q[molecular], batch[molecular], num_graphs)
        for b in periodic.nonzero().flatten().tolist():
            mask = batch == b
            e = self.reciprocal(pos[mask], q[mask], cell[b]).reshape(1)
            out = out.index_put((torch.tensor([b], device=out.device),), e)
        return out


class LatentEwald(InteratomicPotential):
    """Any model plus a LES long-range energy (``model.extra["long_range"]`` in a config).

    Outputs: the wrapped model's keys with ``"energy"`` / ``"node_energy"`` including the
    long-range part (spread evenly over each structure's atoms), plus ``"energy_sr"``,
    ``"energy_lr"``, ``"latent_charges"`` ``(N, n_channels)``, ``"les_charges"`` ``(N,)`` (the
    charge channel in e) and ``"les_dipole"`` ``(B, 3)`` (molecules; zero for periodic cells).
    """

    def __init__(self, model: InteratomicPotential, n_channels: int = 4, hidden=None, q_bias: bool = False,
                 q_add_linear: bool = True, dl: float = 2.0, sigma: float = 1.0, exponent: int = 1,
                 remove_self_interaction: bool = False, constrain_charge: bool = False,
                 charge_channel: int = 0, charge_weights: str = "uniform", charge_solve: bool = False,
                 fragments: bool = False, method: str = "kspace", dipole_origin: str = "com",
                 dielectric: float = 1.0, learn_dielectric: bool = False, **unsupported):
        super().__init__()
        if charge_solve or fragments or method != "kspace":
            raise NotImplementedError("LatentEwald: charge_solve, fragments and method='pme' are not built")
        dim = getattr(model, "node_feature_dim", None)
        if dim is None:
            raise TypeError(f"{type(model).__name__} exposes no node_feature_dim / 'node_features'")
        if not 0 <= charge_channel < n_channels:
            raise ValueError(f"charge_channel must be in [0, {n_channels})")
        if charge_weights not in ("uniform", "learned"):
            raise ValueError("charge_weights must be 'uniform' or 'learned'")
        if dipole_origin not in ("com", "centroid", "origin"):
            raise ValueError("dipole_origin must be 'com', 'centroid' or 'origin'")
        if dielectric <= 0:
            raise ValueError("dielectric must be positive")
        self.model = model
        self.cutoff = model.cutoff
        widths = [dim] + list(hidden or [24, 12])
        layers: List[nn.Module] = []
        for a, b in zip(widths[:-1], widths[1:]):
            layers += [nn.Linear(a, b, bias=q_bias), nn.SiLU()]
        layers.append(nn.Linear(widths[-1], n_channels, bias=q_bias))
        self.q_net = nn.Sequential(*layers)
        self.q_linear = nn.Linear(dim, n_channels, bias=False) if q_add_linear else None
        self.constrain_charge = bool(constrain_charge)
        self.charge_channel = int(charge_channel)
        self.charge_weight = nn.Linear(dim, 1) if constrain_charge and charge_weights == "learned" else None
        self.dipole_origin = dipole_origin
        self.ewald = EwaldSummation(dl=dl, sigma=sigma, exponent=exponent,
                                    remove_self_interaction=remove_self_interaction)
        log_eps = torch.tensor(math.log(float(dielectric)))
        if learn_dielectric:
            self.log_dielectric = nn.Parameter(log_eps)
        else:
            self.register_buffer("log_dielectric", log_eps)
        self.node_feature_dim = dim

    def receptive_field(self) -> Optional[float]:
        return None            # the long-range term couples every atom

    @property
    def dielectric(self) -> Tensor:
        return torch.exp(self.log_dielectric)

    def screened(self, q: Tensor) -> Tensor:
        scale = torch.ones(q.shape[1], dtype=q.dtype, device=q.device)
        scale = scale.index_fill(0, torch.tensor([self.charge_channel], device=q.device),
                                 torch.exp(-0.5 * self.log_dielectric).to(q.dtype))
        return q * scale[None]

    def constrain(self, q: Tensor, features: Tensor, batch: Tensor, num_graphs: int,
                  total_charge: Optional[Tensor]) -> Tensor:
        """Shift each structure's charges so the charge channel sums to its net charge (in
        latent units) and the other channels to zero."""
        target = torch.zeros(num_graphs, q.shape[1], dtype=q.dtype, device=q.device)
        if total_charge is not None:
            target[:, self.charge_channel] = total_charge.to(q.dtype).reshape(-1) * LATENT_CHARGE_PER_E
        if self.charge_weight is not None:
            w = nn.functional.softplus(self.charge_weight(features)).reshape(-1, 1)
        else:
            w = torch.ones(q.shape[0], 1, dtype=q.dtype, device=q.device)
        excess = scatter_sum(q, batch, num_graphs) - target
        wsum = scatter_sum(w, batch, num_graphs)
        return q - w * (excess / wsum)[batch]

    def dipole(self, charges: Tensor, pos: Tensor, data: AtomicGraph, periodic: Tensor) -> Tensor:
        B = data.num_graphs
        if self.dipole_origin == "origin":
            origin = pos.new_zeros(B, 3)
        else:
            if self.dipole_origin == "com":
                w = elements.masses(data.atomic_numbers, pos.dtype)
            else:
                w = torch.ones(pos.shape[0], dtype=pos.dtype, device=pos.device)
            origin = scatter_sum(w[:, None] * pos, data.batch, B) / scatter_sum(w, data.batch, B)[:, None]
        d = scatter_sum(charges[:, None] * (pos - origin[data.batch]), data.batch, B)
        return d * (~periodic).to(d.dtype)[:, None]

    def forward(self, data: AtomicGraph) -> dict:
        out = dict(self.model(data))
        feats = out["node_features"]
        q = self.q_net(feats)
        if self.q_linear is not None:
            q = q + self.q_linear(feats)
        B = data.num_graphs
        if self.constrain_charge:
            q = self.constrain(q, feats, data.batch, B, data.total_charge)
        pos = data.pos.to(q.dtype)
        cell = data.cell.to(q.dtype) if data.cell is not None else None
        e_lr = self.ewald(self.screened(q), pos, data.batch, B, cell, data.pbc)
        e_sr = out["energy"]
        energy = e_sr + e_lr.to(e_sr.dtype)
        counts = torch.bincount(data.batch, minlength=B).clamp(min=1).to(e_lr.dtype)
        node_energy = out["node_energy"] + (e_lr / counts)[data.batch].to(out["node_energy"].dtype)
        periodic = periodic_structures(cell, data.pbc, B, pos.device)
        charges = q[:, self.charge_channel] / LATENT_CHARGE_PER_E
        out.update(energy=energy, node_energy=node_energy, energy_sr=e_sr, energy_lr=e_lr,
                   latent_charges=q, les_charges=charges, les_dipole=self.dipole(charges, pos, data, periodic))
        return out
