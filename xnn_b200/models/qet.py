"""QET (Ko et al., arXiv:2511.07249): TensorNet with analytic charge equilibration.

The TensorNet trunk gives invariant features ``h_i``; an electronegativity network ``chi_i``
(shifted by an external potential when given) and a hardness (one per element, or a softplus
network of ``h_i``) set closed-form charges at the structure's net charge; the charges give a
damped Coulomb potential ``V_i = k_e sum_j q_j erf(r_ij / (sqrt 2 gamma_ij)) f(r_ij) / r_ij`` over
the neighbours (``gamma_ij^2 = sigma_i^2 + sigma_j^2``, covalent radii or learned widths, degree-3
polynomial envelope); the atomic energy is a gated network of the layer-normed
``[h_i, q_i, V_i]``. Defaults and parameter names follow the reference
(``src/xnn/gnn/models/qet.py:112-402``): 32 Gaussians on ``[0, cutoff + 1]`` with exponent 0.5,
no self pairs, gated readout. The charge constraint couples whole structures: no bounded
receptive field.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.blocks import MLP
from ..nn.cutoff import PolynomialCutoff
from ..ops.scatter import scatter_sum
from .charges import closed_form_charges
from .mace import COVALENT_RADII
from .registry import register_model
from .tensornet import TensorNet

COULOMB_CONSTANT = 14.399645478425668
_HARDNESS = ("element", "environment")


class _ElementHardness(nn.Module):
    def __init__(self, n_elements: int):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n_elements))

    def forward(self, x: Tensor, z: Tensor) -> Tensor:
        return self.weight[z]


class _EnvironmentHardness(nn.Module):
    def __init__(self, n_features: int):
        super().__init__()
        self.mlp = MLP([n_features, n_features, n_features, 1], "softplus", activate_last=True)

    def forward(self, x: Tensor, z: Tensor) -> Tensor:
        return self.mlp(x).squeeze(-1)


@register_model("qet")
class QET(TensorNet):
    refreshes_ghosts = False
    readout_extra_inputs = 2

    def __init__(self, n_features: int = 64, n_interactions: int = 2, n_rbf: int = 32, cutoff: float = 5.0,
                 radial_basis: str = "gaussian", trainable_rbf: bool = False, activation: str = "silu",
                 equivariance_group: str = "O(3)", n_elements: int = 128, energy_shift: float = 0.0,
                 energy_scale: float = 1.0, species=None, atomic_energies=None, readout: str = "gated",
                 readout_hidden=None, self_pairs: bool = False, rbf_max: Optional[float] = None,
                 gamma: Optional[float] = None, hardness: str = "element", trainable_widths: bool = False):
        if hardness not in _HARDNESS:
            raise ValueError(f"hardness must be one of {_HARDNESS}, got {hardness!r}")
        if radial_basis == "gaussian":
            rbf_max = float(cutoff) + 1.0 if rbf_max is None else rbf_max
            gamma = 0.5 if gamma is None else gamma
        super().__init__(n_features=n_features, n_interactions=n_interactions, n_rbf=n_rbf, cutoff=cutoff,
                         radial_basis=radial_basis, trainable_rbf=trainable_rbf, activation=activation,
                         equivariance_group=equivariance_group, n_elements=n_elements, energy_shift=energy_shift,
                         energy_scale=energy_scale, species=species, atomic_energies=atomic_energies,
                         readout=readout, readout_hidden=readout_hidden, self_pairs=self_pairs, rbf_max=rbf_max,
                         gamma=gamma)
        self.hardness_mode = hardness
        self.chi_readout = MLP([n_features, n_features, n_features, 1], activation, activate_last=True)
        self.hardness_readout = (_ElementHardness(n_elements) if hardness == "element"
                                 else _EnvironmentHardness(n_features))
        radii = [COVALENT_RADII[z] if z < len(COVALENT_RADII) else 0.2 for z in range(n_elements)]
        if trainable_widths:
            self.sigma = nn.Parameter(torch.ones(n_elements))
        else:
            self.register_buffer("sigma", torch.tensor(radii, dtype=torch.get_default_dtype()))
        self.coulomb_cutoff = PolynomialCutoff(cutoff, p=3)
        self.readout_norm = nn.LayerNorm(n_features + self.readout_extra_inputs)

    def receptive_field(self) -> Optional[float]:
        return None

    def _charge_head(self, x: Tensor, z: Tensor, edge_index: Tensor, vec: Tensor, batch: Tensor, num_graphs: int,
                     total: Tensor, external: Optional[Tensor]):
        chi = self.chi_readout(x).squeeze(-1)
        if external is not None:
            chi = chi + external.to(chi.dtype)
        q = closed_form_charges(chi, 1.0 / self.hardness_readout(x, z), total, batch, num_graphs)
        src, dst = edge_index[0], edge_index[1]
        r = torch.linalg.norm(vec, dim=-1)
        w2 = self.sigma.to(chi.dtype)[z] ** 2
        g = torch.sqrt(w2.index_select(0, src) + w2.index_select(0, dst))
        pair = q.index_select(0, src) * torch.erf(r / (math.sqrt(2.0) * g)) * self.coulomb_cutoff(r) / r
        v = COULOMB_CONSTANT * scatter_sum(pair, dst, x.shape[0])
        h = self.readout_norm(torch.cat([x, q.unsqueeze(-1), v.unsqueeze(-1)], -1))
        return self._energy(h, z), q, v

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        n = atomic_numbers.shape[0]
        zeros = edge_vec.new_zeros(n)
        x = self._features(self.tensors(atomic_numbers, edge_index, edge_vec, zeros))
        batch = torch.zeros(n, dtype=torch.long, device=edge_vec.device)
        e, _, _ = self._charge_head(x, atomic_numbers, edge_index, edge_vec, batch, 1, edge_vec.new_zeros(1), None)
        return x, e

    def forward(self, data: AtomicGraph) -> dict:
        vec = data.edge_vectors()
        X = self.tensors(data.atomic_numbers, data.edge_index, vec, vec.new_zeros(data.num_nodes))
        x = self._features(X)
        total = data.total_charge if data.total_charge is not None else vec.new_zeros(data.num_graphs)
        ne, q, v = self._charge_head(x, data.atomic_numbers, data.edge_index, vec, data.batch, data.num_graphs,
                                     total, data.external_potential)
        return {"node_energy": ne, "energy": self.aggregate_energy(ne, data), "charges": q,
                "electrostatic_potential": v, "node_features": x, "node_tensors": X}

    @classmethod
    def from_config(cls, cfg) -> "QET":
        extra = dict(cfg.extra or {})
        gamma = extra.get("gamma")
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf, cutoff=cfg.cutoff,
                   radial_basis=str(extra.get("radial_basis", "gaussian")),
                   trainable_rbf=bool(extra.get("trainable_rbf", False)),
                   activation=str(extra.get("activation", "silu")),
                   equivariance_group=str(extra.get("equivariance_group", "O(3)")),
                   n_elements=int(extra.get("n_elements", 128)),
                   energy_shift=float(extra.get("energy_shift", 0.0)),
                   energy_scale=float(extra.get("energy_scale", 1.0)), species=extra.get("species"),
                   atomic_energies=extra.get("atomic_energies"), readout=str(extra.get("readout", "gated")),
                   readout_hidden=extra.get("readout_hidden"), self_pairs=bool(extra.get("self_pairs", False)),
                   rbf_max=None if extra.get("rbf_max") is None else float(extra["rbf_max"]),
                   gamma=None if gamma is None else float(gamma), hardness=str(extra.get("hardness", "element")),
                   trainable_widths=bool(extra.get("trainable_widths", False)))
