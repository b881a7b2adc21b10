"""PhysNet (Unke & Meuwly, JCTC 15, 3678, 2019): message passing with per-atom energies and
charges, shielded/switched Coulomb and D3(BJ) dispersion.

Embeddings of ``Z`` (95 rows); radial functions ``phi(r) exp(-beta_k (exp(-r) - mu_k)^2)``
(softplus-reparametrised centres and widths, quintic envelope); ``num_blocks`` modules of an
interaction layer (gated features, message ``sum_j (G g_ij) * dense_j(x_j)``, residual stacks,
``u * x + dense(m)``) and atomic residual stacks, each feeding an output block of energy and
charge; per-element scale/shift tables; charges corrected to the net charge; Coulomb
``k_e/2 q_i q_j [(1-w) / sqrt(r^2+1) + w / r]`` with a quintic switch at ``sr_cut / 2`` (and
force-shifted at ``lr_cut`` when set); learnable-or-fixed D3(BJ); the non-hierarchicality penalty
``nh_loss``. Weights are stored ``(n_in, n_out)`` as in the original code; parameter names follow
the reference (``src/xnn/dnn/models/physnet.py:87-749``) so that weights transplant.
"""
from __future__ import annotations

import math
from typing import List, Optional

import numpy as np
import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.blocks import shifted_softplus
from ..ops.scatter import scatter_sum
from . import d3_legacy
from .base import InteratomicPotential
from .registry import register_model

MAX_Z = 95
KEHALF = 7.199822675975274


def softplus_inverse(x):
    return x + np.log(-np.expm1(-x))


def semi_orthogonal_glorot_weights(n_in: int, n_out: int, scale: float = 2.0) -> Tensor:
    dim = max(n_in, n_out)
    q, r = torch.linalg.qr(torch.randn(dim, dim, dtype=torch.float64))
    w = (q * torch.sign(torch.diagonal(r)))[:n_in, :n_out]
    w = w * torch.sqrt(scale / ((n_in + n_out) * w.var()))
    return w.to(torch.get_default_dtype())


class _Dense(nn.Module):
    def __init__(self, n_in: int, n_out: int, activation: bool = False, use_bias: bool = True,
                 zero_init: bool = False):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(n_in, n_out) if zero_init else semi_orthogonal_glorot_weights(n_in, n_out))
        self.bias = nn.Parameter(torch.zeros(n_out)) if use_bias else None
        self.activation = activation

    def forward(self, x: Tensor) -> Tensor:
        y = torch.addmm(self.bias, x, self.weight) if self.bias is not None else x @ self.weight
        return shifted_softplus(y) if self.activation else y


class _Residual(nn.Module):
    def __init__(self, n: int):
        super().__init__()
        self.dense = _Dense(n, n, activation=True)
        self.residual = _Dense(n, n)

    def forward(self, x: Tensor) -> Tensor:
        return x + self.residual(self.dense(shifted_softplus(x)))


class _RBF(nn.Module):
    def __init__(self, n_rbf: int, cutoff: float):
        super().__init__()
        self.n_rbf, self.cutoff = n_rbf, cutoff
        grid = np.linspace(1.0, np.exp(-cutoff), n_rbf)
        delta = (1.0 - np.exp(-cutoff)) / n_rbf
        dt = torch.get_default_dtype()
        self.centers = nn.Parameter(torch.as_tensor(softplus_inverse(grid), dtype=dt))
        self.widths = nn.Parameter(torch.full((n_rbf,), float(softplus_inverse((0.5 / delta) ** 2)), dtype=dt))

    def cutoff_fn(self, r: Tensor) -> Tensor:
        x = r / self.cutoff
        return torch.where(x < 1, 1 - 6 * x ** 5 + 15 * x ** 4 - 10 * x ** 3, torch.zeros_like(x))

    def forward(self, r: Tensor) -> Tensor:
        r = r.unsqueeze(-1)
        return self.cutoff_fn(r) * torch.exp(-F.softplus(self.widths) * (torch.exp(-r) - F.softplus(self.centers)) ** 2)


class _InteractionLayer(nn.Module):
    def __init__(self, n_rbf: int, n: int, num_residual: int):
        super().__init__()
        self.k2f = _Dense(n_rbf, n, use_bias=False, zero_init=True)
        self.dense_i = _Dense(n, n, activation=True)
        self.dense_j = _Dense(n, n, activation=True)
        self.residuals = nn.ModuleList([_Residual(n) for _ in range(num_residual)])
        self.dense = _Dense(n, n)
        self.u = nn.Parameter(torch.ones(n))

    def forward(self, x: Tensor, rbf: Tensor, edge_index: Tensor) -> Tensor:
        xa = shifted_softplus(x)
        j, i = edge_index[0], edge_index[1]
        m = self.dense_i(xa) + scatter_sum(self.k2f(rbf) * self.dense_j(xa).index_select(0, j), i, x.shape[0])
        for res in self.residuals:
            m = res(m)
        return self.u * x + self.dense(shifted_softplus(m))


class _InteractionBlock(nn.Module):
    def __init__(self, n_rbf: int, n: int, num_residual_atomic: int, num_residual_interaction: int):
        super().__init__()
        self.interaction = _InteractionLayer(n_rbf, n, num_residual_interaction)
        self.residuals = nn.ModuleList([_Residual(n) for _ in range(num_residual_atomic)])

    def forward(self, x: Tensor, rbf: Tensor, edge_index: Tensor) -> Tensor:
        x = self.interaction(x, rbf, edge_index)
        for res in self.residuals:
            x = res(x)
        return x


class _OutputBlock(nn.Module):
    def __init__(self, n: int, num_residual: int):
        super().__init__()
        self.residuals = nn.ModuleList([_Residual(n) for _ in range(num_residual)])
        self.dense = _Dense(n, 2, use_bias=False, zero_init=True)

    def forward(self, x: Tensor) -> Tensor:
        for res in self.residuals:
            x = res(x)
        return self.dense(shifted_softplus(x))


@register_model("physnet")
class PhysNet(InteratomicPotential):
    head_modules = ("output_blocks", "Eshift", "Escale", "Qshift", "Qscale")

    def __init__(self, cutoff: float = 10.0, lr_cutoff: Optional[float] = None, n_features: int = 128, n_rbf: int = 64,
                 num_blocks: int = 5, num_residual_atomic: int = 2, num_residual_interaction: int = 3,
                 num_residual_output: int = 1, use_electrostatics: bool = True, use_dispersion: bool = True,
                 s6: Optional[float] = None, s8: Optional[float] = None, a1: Optional[float] = None,
                 a2: Optional[float] = None, d3_references: str = "2010", energy_shift: float = 0.0,
                 energy_scale: float = 1.0, charge_shift: float = 0.0, charge_scale: float = 1.0, species=None,
                 atomic_energies=None, atomic_scales=None):
        super().__init__()
        if num_blocks < 1:
            raise ValueError("num_blocks must be >= 1")
        self.sr_cut = float(cutoff)
        self.lr_cut = None if lr_cutoff is None else float(lr_cutoff)
        if species is not None:
            self.species = [int(z) for z in species]
        self.cutoff = self.lr_cut if self.lr_cut is not None else self.sr_cut
        self.n_features = n_features
        self.node_feature_dim = n_features
        self.use_electrostatics, self.use_dispersion = use_electrostatics, use_dispersion
        self.embeddings = nn.Parameter(torch.empty(MAX_Z, n_features).uniform_(-math.sqrt(3), math.sqrt(3)))
        self.rbf_layer = _RBF(n_rbf, cutoff)
        self.interaction_blocks = nn.ModuleList([_InteractionBlock(n_rbf, n_features, num_residual_atomic,
                                                                   num_residual_interaction) for _ in range(num_blocks)])
        self.output_blocks = nn.ModuleList([_OutputBlock(n_features, num_residual_output) for _ in range(num_blocks)])
        self.Eshift = nn.Parameter(torch.full((MAX_Z,), float(energy_shift)))
        self.Escale = nn.Parameter(torch.full((MAX_Z,), float(energy_scale)))
        self.Qshift = nn.Parameter(torch.full((MAX_Z,), float(charge_shift)))
        self.Qscale = nn.Parameter(torch.full((MAX_Z,), float(charge_scale)))
        self._learnable = {}
        for name, value, default in (("s6", s6, d3_legacy.S6), ("s8", s8, d3_legacy.S8), ("a1", a1, d3_legacy.A1),
                                     ("a2", a2, d3_legacy.A2)):
            if value is None:
                setattr(self, f"_{name}", nn.Parameter(torch.tensor(float(softplus_inverse(default)))))
            else:
                self.register_buffer(f"_{name}", torch.tensor(float(value)))
            self._learnable[name] = value is None
        if use_dispersion:
            c6ab, rcov, r2r4 = d3_legacy.legacy_tables(str(d3_references))
            dt = torch.get_default_dtype()
            self.register_buffer("_d3_c6ab", c6ab.to(dt), persistent=False)
            self.register_buffer("_d3_rcov", rcov.to(dt), persistent=False)
            self.register_buffer("_d3_r2r4", r2r4.to(dt), persistent=False)
        if atomic_energies is not None or atomic_scales is not None:
            if species is None:
                raise ValueError("species is required to map atomic_energies/atomic_scales")
            with torch.no_grad():
                idx = torch.tensor(list(species))
                if atomic_energies is not None:
                    self.Eshift[idx] = torch.as_tensor(atomic_energies, dtype=self.Eshift.dtype)
                if atomic_scales is not None:
                    self.Escale[idx] = torch.as_tensor(atomic_scales, dtype=self.Escale.dtype)

    def _d3(self, name: str) -> Tensor:
        raw = getattr(self, f"_{name}")
        return F.softplus(raw) if self._learnable[name] else raw

    s6 = property(lambda self: self._d3("s6"))
    s8 = property(lambda self: self._d3("s8"))
    a1 = property(lambda self: self._d3("a1"))
    a2 = property(lambda self: self._d3("a2"))

    def atomic_properties(self, z: Tensor, edge_index: Tensor, edge_vec: Tensor):
        d = torch.linalg.norm(edge_vec, dim=-1)
        rbf = self.rbf_layer(d)
        x = self.embeddings[z]
        energy, charge = x.new_zeros(x.shape[0]), x.new_zeros(x.shape[0])
        sq: List[Tensor] = []
        for inter, head in zip(self.interaction_blocks, self.output_blocks):
            x = inter(x, rbf, edge_index)
            eq = head(x)
            energy = energy + eq[:, 0]
            charge = charge + eq[:, 1]
            sq.append(eq ** 2)
        nh = x.new_zeros(())
        for prev, cur in zip(sq, sq[1:]):
            nh = nh + torch.mean(cur / (cur + prev + 1e-7))
        return self.Escale[z] * energy + self.Eshift[z], self.Qscale[z] * charge + self.Qshift[z], d, nh, x

    def scaled_charges(self, q: Tensor, batch: Tensor, num_graphs: int, total: Optional[Tensor] = None) -> Tensor:
        n_per = scatter_sum(torch.ones_like(q), batch, num_graphs)
        total = q.new_zeros(num_graphs) if total is None else total.to(q.dtype)
        return q + ((total - scatter_sum(q, batch, num_graphs)) / n_per)[batch]

    def _switch(self, d: Tensor) -> Tensor:
        half = self.sr_cut / 2
        y = d / half
        return torch.where(d < half, y ** 3 * (y * (6.0 * y - 15.0) + 10.0), torch.ones_like(d))

    def electrostatic_energy_per_atom(self, d: Tensor, q: Tensor, i: Tensor, j: Tensor) -> Tensor:
        qq = KEHALF * q.index_select(0, i) * q.index_select(0, j)
        rb = torch.sqrt(d * d + 1.0)
        w = self._switch(d)
        if self.lr_cut is None:
            e = qq * ((1.0 - w) / rb + w / d)
        else:
            rc = self.lr_cut
            bare = 1.0 / d + d / rc ** 2 - 2.0 / rc
            bound = 1.0 / rb + rb / rc ** 2 - 2.0 / rc
            e = torch.where(d <= rc, qq * ((1.0 - w) * bound + w * bare), torch.zeros_like(d))
        return scatter_sum(e, i, q.shape[0])

    def dispersion_energy_per_atom(self, z: Tensor, d: Tensor, i: Tensor, j: Tensor) -> Tensor:
        cut = None if self.lr_cut is None else self.lr_cut / d3_legacy.AUTOANG
        return d3_legacy.AUTOEV * d3_legacy.pair_dispersion(
            z, d / d3_legacy.AUTOANG, i, j, cut, self.s6, self.s8, self.a1, self.a2, self._d3_c6ab, self._d3_rcov,
            self._d3_r2r4)

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        j, i = edge_index[0], edge_index[1]
        e, q, d, _, x = self.atomic_properties(atomic_numbers, edge_index, edge_vec)
        q = q - q.sum() / q.shape[0]
        if self.use_electrostatics:
            e = e + self.electrostatic_energy_per_atom(d, q, i, j)
        if self.use_dispersion:
            e = e + self.dispersion_energy_per_atom(atomic_numbers, d, i, j)
        return x, e

    def forward(self, data: AtomicGraph) -> dict:
        j, i = data.edge_index[0], data.edge_index[1]
        e, q, d, nh, x = self.atomic_properties(data.atomic_numbers, data.edge_index, data.edge_vectors())
        q = self.scaled_charges(q, data.batch, data.num_graphs, data.total_charge)
        if self.use_electrostatics:
            e = e + self.electrostatic_energy_per_atom(d, q, i, j)
        if self.use_dispersion:
            e = e + self.dispersion_energy_per_atom(data.atomic_numbers, d, i, j)
        dipole = scatter_sum(q.unsqueeze(-1) * data.pos.to(q.dtype), data.batch, data.num_graphs)
        return {"node_energy": e, "energy": self.aggregate_energy(e, data), "charges": q, "dipole": dipole,
                "nh_loss": nh, "node_features": x}

    @classmethod
    def from_config(cls, cfg) -> "PhysNet":
        e = dict(cfg.extra or {})
        opt = lambda k: None if e.get(k) is None else float(e[k])  # noqa: E731
        return cls(cutoff=cfg.cutoff, lr_cutoff=opt("lr_cutoff"), n_features=cfg.n_features, n_rbf=cfg.n_rbf,
                   num_blocks=cfg.n_interactions, num_residual_atomic=int(e.get("num_residual_atomic", 2)),
                   num_residual_interaction=int(e.get("num_residual_interaction", 3)),
                   num_residual_output=int(e.get("num_residual_output", 1)),
                   use_electrostatics=bool(e.get("use_electrostatics", True)),
                   use_dispersion=bool(e.get("use_dispersion", True)), s6=opt("s6"), s8=opt("s8"), a1=opt("a1"),
                   a2=opt("a2"), d3_references=str(e.get("d3_references", "2010")),
                   energy_shift=float(e.get("energy_shift", 0.0)), energy_scale=float(e.get("energy_scale", 1.0)),
                   charge_shift=float(e.get("charge_shift", 0.0)), charge_scale=float(e.get("charge_scale", 1.0)),
                   species=e.get("species"), atomic_energies=e.get("atomic_energies"),
                   atomic_scales=e.get("atomic_scales"))
