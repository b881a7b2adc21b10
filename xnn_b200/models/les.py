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

With ``charge_solve`` the head's charge channel is an electronegativity ``chi`` and the charges
minimise ``sum chi q + J q^2 / 2 + E_lr(q)`` at the structure's net charge (one augmented solve
per structure, the Coulomb matrix the Hessian of the long-range energy; hardness per element or
from the features); with ``fragments`` there is one constraint per bonded fragment (ions on their
own, charges from ``fragment_charges`` labels or the ion table). ``method="pme"`` evaluates the
reciprocal sum on a smooth-PME mesh (order 8, oversampled twice by default): the same wave-vector
sphere and weights, structure factors from B-spline-spread charges.
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


def smooth_size(n: float) -> int:
    """The smallest integer of at least ``n`` (and 8) with no prime factor above 5."""
    size = max(8, int(math.ceil(n)))
    while True:
        rest = size
        for prime in (2, 3, 5):
            while rest % prime == 0:
                rest //= prime
        if rest == 1:
            return size
        size += 1


class EwaldSummation(nn.Module):
    """Ewald energy of a per-atom latent variable ``q`` (see module notes)."""

    def __init__(self, dl: float = 2.0, sigma: float = 1.0, exponent: int = 1,
                 remove_self_interaction: bool = False, atom_block: int = 4096, method: str = "kspace",
                 pme_order: int = 8, pme_oversample: float = 2.0):
        super().__init__()
        if exponent not in (1, 6):
            raise ValueError(f"exponent must be 1 or 6, got {exponent}")
        if method not in ("kspace", "pme"):
            raise ValueError(f"method must be 'kspace' or 'pme', got {method!r}")
        self.dl, self.sigma, self.exponent = float(dl), float(sigma), int(exponent)
        self.remove_self_interaction = bool(remove_self_interaction)
        self.atom_block = int(atom_block)
        self.method, self.pme_order, self.pme_oversample = method, int(pme_order), float(pme_oversample)

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

    def pme_mesh(self, cell: Tensor) -> List[int]:
        return [smooth_size(2.0 * self.pme_oversample * float(L) / self.dl)
                for L in torch.linalg.norm(cell.detach(), dim=1).tolist()]

    def reciprocal_pme(self, pos: Tensor, q: Tensor, cell: Tensor) -> Tensor:
        """:meth:`reciprocal` with the structure factors from a smooth-PME mesh (full FFT grid)."""
        from ..ffnn.multipoles import bspline_moduli, spread
        mesh = self.pme_mesh(cell)
        axes = [torch.fft.fftfreq(k, d=1.0 / k, dtype=cell.dtype, device=cell.device) for k in mesh]
        miller = torch.stack(torch.meshgrid(*axes, indexing="ij"), -1)
        kvec = 2.0 * math.pi * (miller @ torch.linalg.inv(cell).t())
        k2 = (kvec * kvec).sum(-1)
        inside = (k2 > 0) & (k2 <= (2.0 * math.pi / self.dl) ** 2 * (1.0 + 1e-9))
        weight = torch.where(inside, self.kernel(torch.where(inside, k2, torch.ones_like(k2))),
                             torch.zeros_like(k2)) / cell_volume(cell)
        B = (bspline_moduli(mesh[0], self.pme_order, cell.dtype, cell.device)[:, None, None]
             * bspline_moduli(mesh[1], self.pme_order, cell.dtype, cell.device)[None, :, None]
             * bspline_moduli(mesh[2], self.pme_order, cell.dtype, cell.device)[None, None, :])
        power = 0.0
        for c in range(q.shape[1]):
            F = torch.fft.fftn(spread(pos, cell, q[:, c], None, None, mesh, self.pme_order))
            power = power + F.real.square() + F.imag.square()
        energy = (weight * B * power).sum()
        if self.remove_self_interaction and self.exponent == 1:
            energy = energy - self.self_energy(q)
        return energy

    def coulomb_matrix(self, pos: Tensor, cell: Optional[Tensor] = None) -> Tensor:
        """``gamma`` with ``E_lr(q) = q^T gamma q / 2`` for one structure (exponent 1)."""
        if self.exponent != 1:
            raise ValueError("the charge solve needs the Coulomb kernel (exponent=1)")
        n = pos.shape[0]
        eye = torch.eye(n, dtype=pos.dtype, device=pos.device)
        self_term = 2.0 / (self.sigma * (2.0 * math.pi) ** 1.5)
        if cell is None:
            dist = torch.linalg.norm(pos[:, None, :] - pos[None, :, :], dim=-1)
            gamma = torch.special.erf(dist / (self.sigma * math.sqrt(2.0))) / (dist + 1e-6) / (2.0 * math.pi)
            return gamma if self.remove_self_interaction else gamma + eye * self_term
        _, kpts, k2 = self.wave_vectors(cell)
        w = self.kernel(k2)
        ph = pos @ kpts.T
        c, s = torch.cos(ph), torch.sin(ph)
        gamma = 4.0 / cell_volume(cell) * ((c * w) @ c.T + (s * w) @ s.T)
        return gamma - eye * self_term if self.remove_self_interaction else gamma

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
        if num_graphs == 1:
            recip = self.reciprocal_pme if self.method == "pme" else self.reciprocal
            return recip(pos, q, cell[0]).reshape(1)
        molecular = ~periodic[batch]
        out = self.realspace_batch(pos[molecular], q[molecular], batch[molecular], num_graphs)
        recip = self.reciprocal_pme if self.method == "pme" else self.reciprocal
        for b in periodic.nonzero().flatten().tolist():
            mask = batch == b
            e = recip(pos[mask], q[mask], cell[b]).reshape(1)
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
                 hardness: str = "element", hardness_init: float = 10.0, fragments: bool = False,
                 bond_factor: float = 1.2, ion_charges=None, method: str = "kspace", pme_order: int = 8,
                 pme_oversample: float = 2.0, dipole_origin: str = "com", dielectric: float = 1.0,
                 learn_dielectric: bool = False):
        super().__init__()
        if hardness not in ("element", "features"):
            raise ValueError(f"hardness must be 'element' or 'features', got {hardness!r}")
        if charge_solve and exponent != 1:
            raise ValueError("the charge solve needs the Coulomb kernel (exponent=1)")
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
        self.charge_solve, self.hardness_mode = bool(charge_solve), hardness
        raw0 = math.log(math.expm1(float(hardness_init) / LATENT_CHARGE_PER_E ** 2))   # softplus^-1
        self.hardness_table = self.hardness_net = None
        if charge_solve and hardness == "element":
            self.hardness_table = nn.Embedding(119, 1)
            nn.init.constant_(self.hardness_table.weight, raw0)
        elif charge_solve:
            self.hardness_net = nn.Linear(dim, 1)
            nn.init.zeros_(self.hardness_net.weight)
            nn.init.constant_(self.hardness_net.bias, raw0)
        self.fragments = bool(fragments) and self.charge_solve
        self.bond_factor = float(bond_factor)
        if self.fragments:
            from .charges import ion_charge_table
            from .dispersion import load_tables
            radii = load_tables("d4_reference.npz")["covalent_radius_aa"]
            self.register_buffer("covalent_radii", torch.tensor(radii, dtype=torch.get_default_dtype()),
                                 persistent=False)
            self.register_buffer("ion_charges", ion_charge_table(ion_charges), persistent=False)
        self.ewald = EwaldSummation(dl=dl, sigma=sigma, exponent=exponent,
                                    remove_self_interaction=remove_self_interaction, method=method,
                                    pme_order=pme_order, pme_oversample=pme_oversample)
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

    def hardness_of(self, features: Tensor, z: Tensor) -> Tensor:
        raw = self.hardness_table(z).squeeze(1) if self.hardness_table is not None else \
            self.hardness_net(features).squeeze(1)
        return nn.functional.softplus(raw)

    def solve_charges(self, chi: Tensor, q: Tensor, features: Tensor, data: AtomicGraph, pos: Tensor,
                      cell: Optional[Tensor]):
        """Charges of the charge channel from one augmented solve per structure (see module notes)."""
        from .charges import bonded_fragments, charge_energy, fragment_targets, solve_charges
        batch, B, z = data.batch, data.num_graphs, data.atomic_numbers
        hardness = self.hardness_of(features, z)
        frag_all = None
        if self.fragments:
            frag_all = bonded_fragments(z, data.edge_index, data.edge_vectors().to(pos.dtype),
                                        self.covalent_radii.to(pos.dtype), self.ion_charges.to(pos.dtype),
                                        self.bond_factor)
        solved = torch.zeros_like(chi)
        mus = []
        periodic = periodic_structures(cell, data.pbc, B, pos.device)
        for i in range(B):
            idx = (batch == i).nonzero().flatten()
            gamma = self.ewald.coulomb_matrix(pos[idx], cell[i] if bool(periodic[i]) else None) / \
                self.dielectric.to(chi.dtype)
            total = data.total_charge[i].to(chi.dtype) if data.total_charge is not None else None
            if frag_all is None:
                frag_i = None
                target = total * LATENT_CHARGE_PER_E if total is not None else chi.new_zeros(())
            else:
                frag_i = torch.unique(frag_all[idx], return_inverse=True)[1]
                labeled = data.fragment_charges is not None and (
                    data.fragment_charges_mask is None or bool(data.fragment_charges_mask[i]))
                label = data.fragment_charges[idx].to(chi.dtype) if labeled else None
                target = fragment_targets(frag_i, z[idx], self.ion_charges.to(chi.dtype), label, total) * \
                    LATENT_CHARGE_PER_E
            q_i, mu_i = solve_charges(chi[idx], hardness[idx], gamma, target, frag_i)
            solved = solved.index_copy(0, idx, q_i)
            mus.append(mu_i)
        q = q.clone()
        q[:, self.charge_channel] = solved
        return q, charge_energy(chi, hardness, solved), torch.cat(mus), hardness, frag_all

    def forward(self, data: AtomicGraph) -> dict:
        out = dict(self.model(data))
        feats = out["node_features"]
        q = self.q_net(feats)
        if self.q_linear is not None:
            q = q + self.q_linear(feats)
        B = data.num_graphs
        chi = q[:, self.charge_channel] if self.charge_solve else None
        if self.constrain_charge:
            q = self.constrain(q, feats, data.batch, B, data.total_charge)
        pos = data.pos.to(q.dtype)
        cell = data.cell.to(q.dtype) if data.cell is not None else None
        if chi is not None:
            q, node_qe, mu, hardness, frag = self.solve_charges(chi, q, feats, data, pos, cell)
        e_lr = self.ewald(self.screened(q), pos, data.batch, B, cell, data.pbc)
        e_sr = out["energy"]
        energy = e_sr + e_lr.to(e_sr.dtype)
        counts = torch.bincount(data.batch, minlength=B).clamp(min=1).to(e_lr.dtype)
        node_energy = out["node_energy"] + (e_lr / counts)[data.batch].to(out["node_energy"].dtype)
        periodic = periodic_structures(cell, data.pbc, B, pos.device)
        charges = q[:, self.charge_channel] / LATENT_CHARGE_PER_E
        out.update(energy=energy, node_energy=node_energy, energy_sr=e_sr, energy_lr=e_lr,
                   latent_charges=q, les_charges=charges, les_dipole=self.dipole(charges, pos, data, periodic))
        if chi is not None:
            e_q = scatter_sum(node_qe, data.batch, B)
            out.update(energy_charge=e_q, hardness=hardness, chemical_potential=mu,
                       energy=out["energy"] + e_q.to(out["energy"].dtype),
                       node_energy=out["node_energy"] + node_qe.to(out["node_energy"].dtype))
            if frag is not None:
                out["fragments"] = frag
        return out
