"""Charge equilibration without coupling between the charges (closed form per structure).

The minimum of ``sum_i chi_i q_i + q_i^2 / (2 J_i)`` at a fixed net charge ``Q`` of every
structure is ``q_i = (lambda - chi_i) / J_i`` with ``lambda = (Q + sum chi_j / J_j) / sum 1 / J_j``;
the sum of inverse hardnesses is bounded below by ``1e-12`` (reference
``src/xnn/common/models/charge_solve.py:333``).
"""
from __future__ import annotations

import torch
from torch import Tensor

from ..ops.scatter import scatter_sum


def closed_form_charges(chi: Tensor, inverse_hardness: Tensor, total_charge: Tensor, batch: Tensor,
                        num_graphs: int) -> Tensor:
    sums = scatter_sum(torch.stack([inverse_hardness, chi * inverse_hardness], -1), batch, num_graphs)
    lam = (total_charge.to(chi.dtype) + sums[:, 1]) / sums[:, 0].clamp(min=1e-12)
    return (lam.index_select(0, batch) - chi) * inverse_hardness


def _gaussian_kernel(r: Tensor, iw: Tensor, alpha: float) -> Tensor:
    screen = torch.where(iw > 0, torch.special.erf(r * iw), torch.ones_like(r))
    if alpha > 0:
        screen = screen - torch.special.erf(alpha * r)
    return screen / r


def gaussian_coulomb_matrix(pos: Tensor, sigma: Tensor, cell=None, accuracy: float = 1e-10,
                            background: bool = True) -> Tensor:
    """``A`` with ``E = q^T A q / 2`` for normalised Gaussian charges of widths ``sigma`` (0: point
    charges) of one structure: ``erf(r / (sqrt 2 gamma_ij)) / r`` off the diagonal
    (``gamma_ij^2 = sigma_i^2 + sigma_j^2``), ``1 / (sigma_i sqrt pi)`` on it. A periodic cell is
    Ewald-split at ``alpha = sqrt(pi) (N / V^2)^(1/6)`` with both tails cut below ``accuracy``, and
    ``background`` adds the neutralising term ``-pi / (V alpha^2)`` (reference
    ``src/xnn/common/models/charge_solve.py:181``). Dense, differentiable, ``e^2`` per length."""
    import math
    from .electrostatics import reciprocal_lattice
    n = pos.shape[0]
    s2 = sigma * sigma
    g2 = s2[:, None] + s2[None, :]
    point = g2 <= 0
    iw = torch.where(point, torch.zeros_like(g2), torch.rsqrt(2.0 * torch.where(point, torch.ones_like(g2), g2)))
    self_term = torch.where(sigma > 0, 1.0 / (math.sqrt(math.pi) * torch.where(sigma > 0, sigma, torch.ones_like(sigma))),
                            torch.zeros_like(sigma))
    eye = torch.eye(n, dtype=torch.bool, device=pos.device)
    if cell is None:
        d = pos[:, None, :] - pos[None, :, :]
        r = torch.sqrt(torch.where(eye, torch.ones_like(g2), (d * d).sum(-1)))
        return torch.where(eye, torch.zeros_like(r), _gaussian_kernel(r, iw, 0.0)) + torch.diag(self_term)
    vol = torch.linalg.det(cell).abs()
    root = math.sqrt(-math.log(accuracy))
    alpha = math.sqrt(math.pi) * (n / float(vol.detach()) ** 2) ** (1.0 / 6.0)
    widest = float(torch.sqrt(g2.detach().max() * 2.0)) if bool((~point).any()) else 0.0
    r_cut = max(root / alpha, root * widest)
    inv = torch.linalg.inv(cell)
    d = pos[None, :, :] - pos[:, None, :]
    d = d - torch.round(d.detach() @ inv.detach()) @ cell
    cd = cell.detach()
    spacing = vol.detach() / torch.linalg.norm(torch.linalg.cross(cd[[1, 2, 0]], cd[[2, 0, 1]]), dim=1)
    b = [int(math.ceil(r_cut / float(s))) + 1 for s in spacing]
    shifts = torch.cartesian_prod(*[torch.arange(-k, k + 1, device=pos.device) for k in b]).to(pos.dtype) @ cell
    vec = d[:, :, None, :] + shifts[None, None, :, :]
    rr2 = (vec * vec).sum(-1)
    keep = (rr2.detach() >= 1e-20) & (rr2.detach() <= r_cut * r_cut)
    rr = torch.sqrt(torch.where(keep, rr2, torch.ones_like(rr2)))
    real = torch.where(keep, _gaussian_kernel(rr, iw[:, :, None].expand_as(rr), alpha), torch.zeros_like(rr)).sum(-1)
    _, kvec, k2 = reciprocal_lattice(cell, 2.0 * alpha * root)
    w = 4.0 * math.pi / vol * torch.exp(-k2 / (4.0 * alpha * alpha)) / k2
    ph = pos @ kvec.t()
    c, s = torch.cos(ph), torch.sin(ph)
    amat = real + (c * w) @ c.t() + (s * w) @ s.t() + torch.diag(self_term - 2.0 * alpha / math.sqrt(math.pi))
    if background:
        amat = amat - math.pi / (alpha * alpha) / vol
    return amat


def solve_charges(chi: Tensor, hardness: Tensor, gamma: Tensor, target: Tensor, fragments=None):
    """Minimum of ``chi.q + sum J q^2 / 2 + q^T gamma q / 2`` at fixed net charge (per structure,
    or per fragment): ``(q, mu)`` with ``mu`` the chemical potential of each constraint row.
    The augmented linear system is solved densely; autograd differentiates through the solve."""
    n = chi.shape[0]
    rows = (torch.ones((1, n), dtype=chi.dtype, device=chi.device) if fragments is None
            else torch.nn.functional.one_hot(fragments).to(chi.dtype).t())
    m = rows.shape[0]
    top = torch.cat([gamma + torch.diag(hardness), rows.t()], 1)
    bottom = torch.cat([rows, chi.new_zeros(m, m)], 1)
    rhs = torch.cat([-chi, target.to(chi.dtype).reshape(m)]).unsqueeze(1)
    sol = torch.linalg.solve(torch.cat([top, bottom], 0), rhs)
    return sol[:n, 0], -sol[n:, 0]


#: default ion charges (e) of the fragment constraints: alkali and alkaline-earth cations, zinc, halides
ION_CHARGES = {"Li": 1, "Na": 1, "K": 1, "Rb": 1, "Cs": 1, "Mg": 2, "Ca": 2, "Sr": 2, "Ba": 2, "Zn": 2,
               "F": -1, "Cl": -1, "Br": -1, "I": -1}


def ion_charge_table(ions=None) -> Tensor:
    from ..data.elements import ATOMIC_NUMBERS
    table = torch.zeros(119)
    for key, value in (ION_CHARGES if ions is None else ions).items():
        table[key if isinstance(key, int) else ATOMIC_NUMBERS[str(key)]] = float(value)
    return table


def bonded_fragments(z: Tensor, edge_index: Tensor, edge_vec: Tensor, radii: Tensor, ions: Tensor,
                     bond_factor: float = 1.2) -> Tensor:
    """Connected components of the bond graph (``r < bond_factor (R_i + R_j)``, ions never bonded),
    numbered by their lowest atom index in order."""
    n = z.shape[0]
    src, dst = edge_index[0], edge_index[1]
    bonded = torch.linalg.norm(edge_vec, dim=-1) < bond_factor * (radii[z[src]] + radii[z[dst]])
    is_ion = ions[z] != 0
    keep = bonded & ~is_ion[src] & ~is_ion[dst]
    src, dst = src[keep], dst[keep]
    labels = torch.arange(n, device=z.device)
    for _ in range(n):                      # min-label propagation to a fixed point
        new = labels.scatter_reduce(0, dst, labels[src], reduce="amin", include_self=True)
        if torch.equal(new, labels):
            break
        labels = new
    roots = torch.zeros(n, dtype=torch.long, device=z.device).index_fill(0, labels, 1)
    return (torch.cumsum(roots, 0) - 1)[labels]


def fragment_targets(fragments: Tensor, z: Tensor, ions: Tensor, label=None, total_charge=None) -> Tensor:
    """Net charge of every fragment: its ``fragment_charges`` label (one value per fragment) or
    the sum of its ion charges; checked against the structure's total charge."""
    n_frag = int(fragments.max()) + 1
    if label is not None:
        hi = torch.full((n_frag,), -float("inf"), dtype=label.dtype, device=label.device)
        lo = torch.full((n_frag,), float("inf"), dtype=label.dtype, device=label.device)
        hi = hi.scatter_reduce(0, fragments, label, reduce="amax")
        lo = lo.scatter_reduce(0, fragments, label, reduce="amin")
        if float((hi - lo).abs().max()) > 1e-6:
            raise ValueError("fragment_charges differ between atoms of one fragment (the label is the charge of "
                             "the fragment each atom belongs to; ions are fragments of their own)")
        targets = hi
    else:
        targets = torch.zeros(n_frag, dtype=ions.dtype, device=fragments.device).index_add(0, fragments, ions[z])
    if total_charge is not None and abs(float(targets.sum()) - float(total_charge)) > 1e-6:
        raise ValueError(f"the fragment charges add up to {float(targets.sum()):g} e but the structure's "
                         f"total_charge is {float(total_charge):g} e; label the charged fragments with "
                         "fragment_charges, or name the ions in ion_charges")
    return targets


def charge_energy(chi: Tensor, hardness: Tensor, q: Tensor) -> Tensor:
    """Per-atom ``chi q + J q^2 / 2``."""
    return chi * q + 0.5 * hardness * q * q
