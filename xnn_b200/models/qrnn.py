"""QRNN (Jacobson et al., JCTC 18, 2354, 2022): a charge-aware ANI.

Atoms carry the AEV and a charge-weighted radial vector ``G^qR_i = sum_j q_j g(r_ij)`` on the
AEV's radial grid. Effective electronegativities are predicted recursively by per-element
networks on ``[G^AEV, q, G^qR]`` and turned into closed-form charges at the net charge with the
diagonal EEQ hardnesses of D4 (``charge_model="recursive"``), or (QeqNN, ``"qeq"``) networks
give ``chi = X^2`` and Gaussian widths ``sigma_0 + S^2`` for a full charge equilibration. The
energy adds per-element networks on ``[G^AEV, q, G^qR]``, a sigmoid-attenuated Coulomb sum over
every pair of a molecule and the wB97X-D dispersion on Grimme's D2 ``C6`` and radii. Options,
defaults and parameter names follow the reference (``src/xnn/dnn/models/qrnn.py:190-623``).
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
from torch import Tensor

from ..data import AtomicGraph
from ..featurizers.aev import AEV
from ..ops.scatter import scatter_sum
from .charges import closed_form_charges, gaussian_coulomb_matrix, solve_charges
from .descriptor import DescriptorPotential, ElementNetworks
from .dispersion import HARTREE, load_tables
from .electrostatics import COULOMB_CONSTANT, all_pairs, coulomb_direct
from .registry import register_model

QRNN_SPECIES = [1, 6, 7, 8, 9, 15, 16, 17]
# Grimme, J. Comput. Chem. 27, 1787 (2006), Table 1, H to Xe: C6 (J nm^6 / mol) and R0 (A)
D2_C6 = (0.14, 0.08, 1.61, 1.61, 3.13, 1.75, 1.23, 0.70, 0.75, 0.63, 5.71, 5.71, 10.79, 9.23, 7.84, 5.57, 5.07, 4.61,
         10.80, 10.80, 10.80, 10.80, 10.80, 10.80, 10.80, 10.80, 10.80, 10.80, 10.80, 10.80, 16.99, 17.10, 16.37,
         12.64, 12.47, 12.01, 24.67, 24.67, 24.67, 24.67, 24.67, 24.67, 24.67, 24.67, 24.67, 24.67, 24.67, 24.67,
         37.32, 38.71, 38.44, 31.74, 31.50, 29.99)
D2_R0 = (1.001, 1.012, 0.825, 1.408, 1.485, 1.452, 1.397, 1.342, 1.287, 1.243, 1.144, 1.364, 1.639, 1.716, 1.705,
         1.683, 1.639, 1.595, 1.485, 1.474) + (1.562,) * 10 + (1.650, 1.727, 1.760, 1.771, 1.749, 1.727, 1.628,
         1.606) + (1.639,) * 10 + (1.672, 1.804, 1.881, 1.892, 1.892, 1.881)
C6_UNIT = 1.0e6 / (6.02214076e23 * 1.602176634e-19)    # J nm^6 / mol in eV A^6
_N_Z = 119


def eeq_hardness(species: Sequence[int]) -> list:
    """Diagonal EEQ hardnesses of D4, ``J_A + sqrt(2/pi) / a_A`` in eV per ``e^2``."""
    ref = load_tables("d4_reference.npz")
    eta, rad = ref["eeq_eta"], ref["eeq_rad"]
    return [float((eta[z] + math.sqrt(2.0 / math.pi) / rad[z]) * HARTREE) for z in species]


def chai_head_gordon_dispersion(z: Tensor, pos: Tensor, batch: Tensor, c6: Tensor, r0: Tensor, s6: float,
                                damping: float) -> Tensor:
    """Per-atom ``-s6/2 sum_j sqrt(C6_i C6_j) / r^6 / (1 + a (r / (R0_i + R0_j))^-12)`` (eV, float64)."""
    row, col = all_pairs(batch)
    zr, zc = z[row], z[col]
    d = pos.index_select(0, row) - pos.index_select(0, col)
    r2 = (d * d).sum(-1)
    r0ij = r0[zr] + r0[zc]
    pair = (-0.5 * s6) * torch.sqrt(c6[zr] * c6[zc]) / (1.0 + damping * (r0ij * r0ij / r2) ** 6) / (r2 * r2 * r2)
    return scatter_sum(pair.to(torch.float64), row, z.shape[0])


@register_model("qrnn")
class QRNN(DescriptorPotential):
    def __init__(self, species: Sequence[int] = QRNN_SPECIES, radial_cutoff: float = 5.2, angular_cutoff: float = 3.5,
                 hidden=(128, 128, 64), charge_hidden=None, activation: str = "gelu", atomic_energies=None,
                 aev_kwargs: Optional[dict] = None, charge_model: str = "recursive", n_iterations: int = 2,
                 initial_charges: str = "uniform", hardness: Optional[Sequence[float]] = None,
                 min_width: float = 0.05, coulomb: bool = True, coulomb_midpoint: float = 2.2,
                 coulomb_steepness: float = 8.5, dispersion: bool = True, dispersion_s6: float = 1.0,
                 dispersion_damping: float = 6.0):
        if charge_model not in ("recursive", "qeq"):
            raise ValueError(f"charge_model must be 'recursive' or 'qeq', got {charge_model!r}")
        if initial_charges not in ("uniform", "zero"):
            raise ValueError(f"initial_charges must be 'uniform' or 'zero', got {initial_charges!r}")
        if int(n_iterations) < 1:
            raise ValueError(f"n_iterations must be at least 1, got {n_iterations}")
        species = [int(z) for z in species]
        if dispersion and max(species) > len(D2_C6):
            raise ValueError(f"the dispersion parameters cover H to Xe; got {species}; set dispersion=False")
        aev = AEV(species, radial_cutoff=radial_cutoff, angular_cutoff=angular_cutoff, **(aev_kwargs or {}))
        n_charge = int(aev.radial.etas.numel() * aev.radial.rs.numel())
        super().__init__(aev, species, hidden, activation=activation, atomic_energies=atomic_energies,
                         extra_inputs=1 + n_charge)
        self.n_charge_features = n_charge
        self.charge_model, self.n_iterations, self.initial_charges = charge_model, int(n_iterations), initial_charges
        widths = hidden if charge_hidden is None else charge_hidden
        self.charge_nets = (ElementNetworks(species, aev.output_dim, widths, activation, extra_inputs=1 + n_charge)
                            if charge_model == "recursive"
                            else ElementNetworks(species, aev.output_dim, widths, activation, n_outputs=2))
        values = eeq_hardness(species) if hardness is None else [float(h) for h in hardness]
        if len(values) != len(species):
            raise ValueError(f"hardness: got {len(values)} values for {len(species)} species")
        if min(values) <= 0.0:
            raise ValueError(f"hardness must be positive, got {values}")
        dt = torch.get_default_dtype()
        inv = torch.zeros(_N_Z, dtype=torch.float64)
        for z, h in zip(species, values):
            inv[z] = 1.0 / h
        self.register_buffer("_inverse_hardness_by_z", inv.to(dt), persistent=False)
        self.min_width = float(min_width)
        self.coulomb, self.coulomb_midpoint, self.coulomb_steepness = bool(coulomb), float(coulomb_midpoint), float(
            coulomb_steepness)
        self.dispersion, self.dispersion_s6, self.dispersion_damping = bool(dispersion), float(dispersion_s6), float(
            dispersion_damping)
        c6 = torch.zeros(_N_Z, dtype=torch.float64)
        r0 = torch.ones(_N_Z, dtype=torch.float64)
        for z in range(1, len(D2_C6) + 1):
            c6[z] = D2_C6[z - 1] * C6_UNIT
            r0[z] = D2_R0[z - 1]
        self.register_buffer("_c6_by_z", c6.to(dt), persistent=False)
        self.register_buffer("_r0_by_z", r0.to(dt), persistent=False)
        self.ewald_accuracy = 1e-10

    def receptive_field(self) -> Optional[float]:
        return None

    def _charge_features(self, basis: Tensor, q: Tensor, edge_index: Tensor, n: int) -> Tensor:
        return scatter_sum(basis * q.index_select(0, edge_index[0]).unsqueeze(-1), edge_index[1], n)

    def _qeq_charges(self, chi, sigma, pos, batch, num_graphs, total, cell, periodic):
        q = torch.zeros_like(chi)
        for b in range(num_graphs):
            idx = torch.nonzero(batch == b).flatten()
            box = cell[b].to(chi.dtype) if cell is not None and bool(periodic[b]) else None
            a = COULOMB_CONSTANT * gaussian_coulomb_matrix(pos[idx].to(chi.dtype), sigma[idx], box, self.ewald_accuracy)
            q = q.index_copy(0, idx, solve_charges(chi[idx], torch.zeros_like(chi[idx]), a, total[b].reshape(1))[0])
        return q

    def compute(self, z: Tensor, edge_index: Tensor, edge_vec: Tensor, pos: Tensor, batch: Tensor, num_graphs: int,
                total_charge: Tensor, cell=None, pbc=None) -> dict:
        n = z.shape[0]
        desc = self.featurizer.compute(z, edge_index, edge_vec, n)
        dt = desc.dtype
        r = torch.linalg.norm(edge_vec, dim=-1)
        rad = self.featurizer.radial
        basis = rad.edge_terms(r, rad.prefactor * rad.cutoff_fn(r))
        total = total_charge.to(dt)
        periodic = pbc.any(dim=1) if pbc is not None else torch.zeros(num_graphs, dtype=torch.bool, device=z.device)
        plan = self.element_nets.plan(z)
        if self.charge_model == "recursive":
            inverse = self._inverse_hardness_by_z.to(dt)[z]
            if self.initial_charges == "uniform":
                counts = scatter_sum(torch.ones_like(desc[:, 0]), batch, num_graphs)
                q = (total / counts).index_select(0, batch)
            else:
                q = torch.zeros_like(desc[:, 0])
            chi = torch.zeros_like(q)
            for _ in range(self.n_iterations):
                inputs = torch.cat([q.unsqueeze(-1), self._charge_features(basis, q, edge_index, n)], -1)
                chi = self.charge_nets(desc, z, inputs, plan)
                q = closed_form_charges(chi, inverse, total, batch, num_graphs)
        else:
            xs = self.charge_nets(desc, z, None, plan)
            chi = xs[:, 0] * xs[:, 0]
            q = self._qeq_charges(chi, self.min_width + xs[:, 1] * xs[:, 1], pos, batch, num_graphs, total, cell,
                                  periodic)
        inputs = torch.cat([q.unsqueeze(-1), self._charge_features(basis, q, edge_index, n)], -1)
        short = self.element_nets(desc, z, inputs, plan) + self._self_energies_by_z.to(dt)[z]
        elec = torch.zeros(n, dtype=torch.float64, device=z.device)
        disp = torch.zeros(n, dtype=torch.float64, device=z.device)
        if self.coulomb or self.dispersion:
            if bool(periodic.any()):
                raise ValueError("the QRNN Coulomb and dispersion terms sum every pair of a molecule; periodic "
                                 "structures need coulomb=False and dispersion=False")
            p = pos.to(dt)
            if self.coulomb:
                elec = coulomb_direct(q, p, batch, COULOMB_CONSTANT, self.coulomb_midpoint, self.coulomb_steepness)
            if self.dispersion:
                disp = chai_head_gordon_dispersion(z, p, batch, self._c6_by_z.to(dt), self._r0_by_z.to(dt),
                                                   self.dispersion_s6, self.dispersion_damping)
        node = short + elec + disp if (self.coulomb or self.dispersion) else short
        return {"node_energy": node, "charges": q, "electronegativities": chi, "node_energy_short": short,
                "node_energy_elec": elec, "node_energy_dispersion": disp, "node_features": desc}

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        if self.coulomb or self.dispersion or self.charge_model != "recursive":
            raise RuntimeError("QRNN with Coulomb, dispersion or QeqNN charges needs positions and whole structures")
        n = atomic_numbers.shape[0]
        out = self.compute(atomic_numbers, edge_index, edge_vec, edge_vec.new_zeros(n, 3),
                           torch.zeros(n, dtype=torch.long, device=edge_vec.device), 1, edge_vec.new_zeros(1))
        return out["node_features"], out["node_energy"]

    def forward(self, data: AtomicGraph) -> dict:
        vec = data.edge_vectors()
        total = data.total_charge if data.total_charge is not None else vec.new_zeros(data.num_graphs)
        out = self.compute(data.atomic_numbers, data.edge_index, vec, data.pos, data.batch, data.num_graphs, total,
                           data.cell, data.pbc)
        for k in ("", "_short", "_elec", "_dispersion"):
            out["energy" + k] = self.aggregate_energy(out["node_energy" + k], data)
        if data.pbc is None or not bool(data.pbc.any()):
            q = out["charges"]
            out["dipole"] = scatter_sum(q.unsqueeze(-1) * data.pos.to(q.dtype), data.batch, data.num_graphs)
        return out

    @classmethod
    def from_config(cls, cfg) -> "QRNN":
        e = dict(cfg.extra or {})
        keys = ("species", "angular_cutoff", "hidden", "charge_hidden", "activation", "atomic_energies", "aev_kwargs",
                "charge_model", "n_iterations", "initial_charges", "hardness", "min_width", "coulomb",
                "coulomb_midpoint", "coulomb_steepness", "dispersion", "dispersion_s6", "dispersion_damping")
        kw = {k: e[k] for k in keys if k in e}
        return cls(radial_cutoff=float(e.get("radial_cutoff", cfg.cutoff)), **kw)
