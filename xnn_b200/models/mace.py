"""MACE (Batatia et al. 2022): higher-body-order equivariant message passing.

Architecture, options and state-dict names follow the reference
(``src/xnn/gnn/models/mace.py:740-1796``): a one-hot species embedding, ``T``
interactions of ``linear_up -> radial-MLP-weighted uvu tensor product with the edge
spherical harmonics -> sum over neighbours -> linear / avg_num_neighbors``, a
per-element symmetric contraction of correlation order ``nu``, a linear map plus the
species self-connection, and per-layer readouts (gated MLP on the last one);
``E_i = E0[Z_i] + scale * sum(readouts) + shift``.

Two implementations share the parameters:

* the reference path (any irreps) built on :mod:`xnn_b200.o3`, which runs anywhere
  and is the float64 oracle;
* the fused path (scalar hidden features, ``max_ell <= 3``, ``correlation <= 3``),
  which runs the per-edge and per-atom hot ops as the sm_100a kernels of
  :mod:`xnn_b200.ops.mace_ops` -- fused edge geometry, radial MLP, the gather-product-
  scatter convolution and the symmetric contraction -- each with explicit first and
  second derivatives, so force training never materialises per-edge messages.

``use_fast`` picks between them: ``"auto"`` (fused on CUDA when the model is
eligible), ``True`` (fused wherever eligible, CPU included via the torch twins of the
kernels) or ``False``.
"""
from __future__ import annotations

import ast
import math
from typing import List, Optional, Tuple, Union

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from ..data.elements import COVALENT_RADII
from ..data import AtomicGraph
from ..nn import BesselRBF, GaussianRBF, PolynomialCutoff
from ..o3 import (FullyConnectedNet, FullyConnectedTensorProduct, Irreps, Linear,
                  SphericalHarmonics, TensorProduct, normalize2mom)
from ..ops.scatter import refresh_ghosts, scatter_sum
from .base import GNNPotential
from .fast import AutoPolicy, choose, resolve_use_fast
from .mace_blocks import (ReshapeIrreps, SymmetricContraction, hidden_irreps,
                          tp_out_irreps_with_instructions)
from .registry import register_model

GATES = {"silu": F.silu, "tanh": torch.tanh, "abs": torch.abs, "None": None, None: None}


class ScalarActivation(nn.Module):
    """Second-moment-normalised activation on all-scalar irreps (e3nn ``Activation``)."""

    def __init__(self, irreps, act):
        super().__init__()
        if Irreps(irreps).lmax > 0:
            raise ValueError("gate activation needs all-scalar irreps")
        self.act = normalize2mom(act) if act is not None else None

    def forward(self, x: Tensor) -> Tensor:
        return self.act(x) if self.act is not None else x


class EdgeEmbedding(nn.Module):
    """Spherical harmonics of the edge direction and Bessel (or Gaussian) x polynomial envelope."""

    def __init__(self, l_max: int, n_rbf: int, cutoff: float, p: int = 6, radial_type: str = "bessel",
                 trainable_rbf: bool = False, rbf_prefactor: Optional[float] = None):
        super().__init__()
        self.l_max, self.n_rbf, self.cutoff = l_max, n_rbf, float(cutoff)
        self.irreps_sh = Irreps.spherical_harmonics(l_max)
        self.sph = SphericalHarmonics(self.irreps_sh, normalize=True, normalization="component")
        if radial_type == "bessel":
            self.rbf = BesselRBF(n_rbf, cutoff, trainable=trainable_rbf, prefactor=rbf_prefactor)
        elif radial_type == "gaussian":
            self.rbf = GaussianRBF(n_rbf, cutoff)
        else:
            raise ValueError(f"unknown radial_type {radial_type!r}")
        self.radial_type = radial_type
        self.envelope = PolynomialCutoff(cutoff, p=p)

    def forward(self, vec: Tensor):
        length = torch.linalg.norm(vec, dim=-1)
        return length, self.sph(vec), self.rbf(length) * self.envelope(length)[:, None]


class InteractionBase(nn.Module):
    def __init__(self, node_attrs_irreps, node_feats_irreps, edge_attrs_irreps, edge_feats_irreps,
                 target_irreps, hidden_irreps_, avg_num_neighbors, radial_MLP):
        super().__init__()
        self.node_attrs_irreps = Irreps(node_attrs_irreps)
        self.node_feats_irreps = Irreps(node_feats_irreps)
        self.edge_attrs_irreps = Irreps(edge_attrs_irreps)
        self.edge_feats_irreps = Irreps(edge_feats_irreps)
        self.target_irreps = Irreps(target_irreps)
        self.hidden_irreps = Irreps(hidden_irreps_)
        self.avg_num_neighbors = float(avg_num_neighbors)
        self.radial_MLP = list(radial_MLP)
        self.linear_up = Linear(self.node_feats_irreps, self.node_feats_irreps)
        irreps_mid, instructions = tp_out_irreps_with_instructions(
            self.node_feats_irreps, self.edge_attrs_irreps, self.target_irreps)
        self.conv_tp = TensorProduct(self.node_feats_irreps, self.edge_attrs_irreps, irreps_mid,
                                     instructions, shared_weights=False, internal_weights=False)
        self.conv_tp_weights = FullyConnectedNet(
            [self.edge_feats_irreps.num_irreps] + self.radial_MLP + [self.conv_tp.weight_numel], F.silu)
        self.irreps_out = self.target_irreps
        self.linear = Linear(irreps_mid, self.irreps_out)
        self.reshape = ReshapeIrreps(self.irreps_out)
        self._setup()

    residual = False
    density = False

    def _setup(self):  # pragma: no cover - overridden
        raise NotImplementedError

    def messages(self, feats: Tensor, edge_attrs: Tensor, edge_feats: Tensor, edge_index: Tensor,
                 n_atoms: int) -> Tensor:
        w = self.conv_tp_weights(edge_feats)
        msg = self.conv_tp(feats.index_select(0, edge_index[0]), edge_attrs, w)
        return scatter_sum(msg, edge_index[1], n_atoms)

    def forward(self, node_attrs, node_feats, edge_attrs, edge_feats, edge_index):
        n = node_feats.shape[0]
        sc = self.skip_tp(node_feats, node_attrs) if self.residual else None
        feats = self.linear_up(node_feats)
        pooled = self.messages(feats, edge_attrs, edge_feats, edge_index, n)
        if self.density:
            rho = scatter_sum(torch.tanh(self.density_fn(edge_feats) ** 2), edge_index[1], n)
            pooled = self.linear(pooled) / (rho + 1.0)
        else:
            pooled = self.linear(pooled) / self.avg_num_neighbors
        if not self.residual:
            pooled = self.skip_tp(pooled, node_attrs)
        return self.reshape(pooled), sc


class RealAgnosticInteractionBlock(InteractionBase):
    """Non-residual: the species self-connection acts on the aggregated message."""

    def _setup(self):
        self.skip_tp = FullyConnectedTensorProduct(self.irreps_out, self.node_attrs_irreps, self.irreps_out)


class RealAgnosticResidualInteractionBlock(InteractionBase):
    """Residual: the self-connection of the input features is added after the product."""

    residual = True

    def _setup(self):
        self.skip_tp = FullyConnectedTensorProduct(self.node_feats_irreps, self.node_attrs_irreps,
                                                   self.hidden_irreps)


class RealAgnosticDensityInteractionBlock(RealAgnosticInteractionBlock):
    """Non-residual, messages divided by ``1 + sum_j tanh(d(e_ij)^2)`` (MACE-MP density generation)."""

    density = True

    def _setup(self):
        super()._setup()
        self.density_fn = FullyConnectedNet([self.edge_feats_irreps.num_irreps, 1], F.silu)


class RealAgnosticDensityResidualInteractionBlock(RealAgnosticResidualInteractionBlock):
    density = True

    def _setup(self):
        super()._setup()
        self.density_fn = FullyConnectedNet([self.edge_feats_irreps.num_irreps, 1], F.silu)


INTERACTIONS = {
    "RealAgnosticInteractionBlock": RealAgnosticInteractionBlock,
    "RealAgnosticResidualInteractionBlock": RealAgnosticResidualInteractionBlock,
    "RealAgnosticDensityInteractionBlock": RealAgnosticDensityInteractionBlock,
    "RealAgnosticDensityResidualInteractionBlock": RealAgnosticDensityResidualInteractionBlock,
}


class EquivariantProductBasis(nn.Module):
    def __init__(self, node_feats_irreps, target_irreps, correlation: int, num_elements: int,
                 use_sc: bool = True):
        super().__init__()
        self.use_sc = use_sc
        self.symmetric_contractions = SymmetricContraction(node_feats_irreps, target_irreps,
                                                           correlation, num_elements)
        self.linear = Linear(target_irreps, target_irreps)

    def forward(self, node_feats: Tensor, sc: Optional[Tensor], node_attrs: Tensor) -> Tensor:
        out = self.linear(self.symmetric_contractions(node_feats, node_attrs))
        if self.use_sc and sc is not None:
            return out + sc
        return out


class ScaleShift(nn.Module):
    def __init__(self, scale: float = 1.0, shift: float = 0.0):
        super().__init__()
        self.register_buffer("scale", torch.tensor(float(scale)))
        self.register_buffer("shift", torch.tensor(float(shift)))

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        for n in ("scale", "shift"):
            if prefix + n not in state_dict:
                state_dict[prefix + n] = getattr(self, n).detach().clone()
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def forward(self, x: Tensor) -> Tensor:
        return self.scale * x + self.shift


class LinearReadout(nn.Module):
    def __init__(self, irreps_in, irrep_out="1x0e"):
        super().__init__()
        self.linear = Linear(irreps_in, irrep_out)

    def forward(self, x: Tensor) -> Tensor:
        return self.linear(x)


class NonLinearReadout(nn.Module):
    def __init__(self, irreps_in, MLP_irreps, gate, irrep_out="1x0e"):
        super().__init__()
        self.linear_1 = Linear(irreps_in, MLP_irreps)
        self.non_linearity = ScalarActivation(MLP_irreps, gate)
        self.linear_2 = Linear(MLP_irreps, irrep_out)

    def forward(self, x: Tensor) -> Tensor:
        return self.linear_2(self.non_linearity(self.linear_1(x)))


class ZBLPairRepulsion(nn.Module):
    """Ziegler-Biersack-Littmark screened Coulomb repulsion tapered at the covalent-radii sum."""

    def __init__(self, p: int = 6):
        super().__init__()
        self.register_buffer("c", torch.tensor([0.1818, 0.5099, 0.2802, 0.02817]))
        self.register_buffer("p", torch.tensor(p, dtype=torch.int))
        radii = COVALENT_RADII + [1.5] * (120 - len(COVALENT_RADII))
        self.register_buffer("covalent_radii", torch.tensor(radii))
        self.register_buffer("a_exp", torch.tensor(0.300))
        self.register_buffer("a_prefactor", torch.tensor(0.4543))

    def forward(self, lengths: Tensor, atomic_numbers: Tensor, edge_index: Tensor, n: int) -> Tensor:
        r = lengths
        zs = atomic_numbers[edge_index[0]].to(r.dtype).unsqueeze(-1)
        zd = atomic_numbers[edge_index[1]].to(r.dtype).unsqueeze(-1)
        a = self.a_prefactor * 0.529 / (zs ** self.a_exp + zd ** self.a_exp)
        d = r / a
        c = self.c
        phi = (c[0] * torch.exp(-3.2 * d) + c[1] * torch.exp(-0.9423 * d)
               + c[2] * torch.exp(-0.4028 * d) + c[3] * torch.exp(-0.2016 * d))
        e = 14.3996 * zs * zd / r * phi
        rc = (self.covalent_radii[atomic_numbers[edge_index[0]]]
              + self.covalent_radii[atomic_numbers[edge_index[1]]]).unsqueeze(-1)
        p = self.p.to(r.dtype)
        s = r / rc
        env = (1.0 - (p + 1) * (p + 2) / 2 * s ** p + p * (p + 2) * s ** (p + 1)
               - p * (p + 1) / 2 * s ** (p + 2)) * (r < rc)
        return scatter_sum(0.5 * e * env, edge_index[1], n).squeeze(-1)


@register_model("mace")
class MACE(GNNPotential):
    head_modules = ("readouts", "atom_ref", "scale_shift")
    refreshes_ghosts = True

    def __init__(self, species, cutoff: float = 4.0, max_ell: int = 3, max_L: int = 0,
                 num_channels: int = 32, n_rbf: int = 8, num_interactions: int = 2,
                 correlation: Union[int, List[int]] = 3, MLP_irreps: str = "16x0e",
                 radial_MLP: Optional[List[int]] = None,
                 interaction: str = "RealAgnosticResidualInteractionBlock",
                 interaction_first: str = "RealAgnosticResidualInteractionBlock",
                 gate: Optional[str] = "silu", avg_num_neighbors: float = 1.0,
                 hidden_irreps: Optional[str] = None, num_cutoff_basis: int = 5,
                 radial_type: str = "bessel", distance_transform: str = "None",
                 pair_repulsion: bool = False, atomic_energies=None, scale: float = 1.0,
                 shift: float = 0.0, rbf_prefactor: Optional[float] = None):
        if num_interactions < 0:
            raise ValueError("num_interactions (T) must be >= 0")
        if distance_transform not in ("None", None):
            from ..nn.transforms import DISTANCE_TRANSFORMS
            if distance_transform not in DISTANCE_TRANSFORMS:
                raise NotImplementedError(f"distance_transform={distance_transform!r}")
        super().__init__(species, cutoff)
        self.max_ell, self.max_L, self.n_rbf = max_ell, max_L, n_rbf
        self.node_attr_irreps = Irreps([(len(self.species), "0e")])
        self.edge_feat = EdgeEmbedding(max_ell, n_rbf, cutoff, p=num_cutoff_basis,
                                       radial_type=radial_type, rbf_prefactor=rbf_prefactor)
        self.irreps_sh = self.edge_feat.irreps_sh
        if atomic_energies is not None:
            self.set_atomic_energies(atomic_energies)
        if distance_transform in ("None", None):
            self.distance_transform = None
        else:
            from ..nn.transforms import DISTANCE_TRANSFORMS
            self.distance_transform = DISTANCE_TRANSFORMS[distance_transform]()
        self.scale_shift = ScaleShift(scale, shift)
        num_elements = len(self.species)
        hid = Irreps(hidden_irreps) if hidden_irreps is not None else _hidden(num_channels, max_L)
        MLP_irreps = Irreps(MLP_irreps)
        radial_MLP = list(radial_MLP) if radial_MLP is not None else [64, 64, 64]
        if isinstance(correlation, int):
            correlation = [correlation] * max(num_interactions, 1)
        self.correlation = list(correlation)
        gate_fn = GATES[gate]
        num_features = hid.count("0e")
        node_feats_irreps = Irreps([(num_features, "0e")])
        self.num_features = num_features
        self._n_scalar_features = num_features
        self.node_feature_dim = num_features * max(1, num_interactions)
        interaction_irreps = hidden_irreps_of(num_features, max_ell)
        edge_feats_irreps = Irreps(f"{n_rbf}x0e")
        self.node_embedding = Linear(self.node_attr_irreps, node_feats_irreps)
        self.pair_repulsion = bool(pair_repulsion)
        if pair_repulsion:
            self.pair_repulsion_fn = ZBLPairRepulsion(p=num_cutoff_basis)
        self.interactions = nn.ModuleList()
        self.products = nn.ModuleList()
        self.readouts = nn.ModuleList()
        self.interaction_names = (interaction_first, interaction)
        if num_interactions >= 1:
            hidden_out = Irreps(str(hid[0])) if num_interactions == 1 else hid
            self.interactions.append(INTERACTIONS[interaction_first](
                self.node_attr_irreps, node_feats_irreps, self.irreps_sh, edge_feats_irreps,
                interaction_irreps, hidden_out, avg_num_neighbors, radial_MLP))
            self.products.append(EquivariantProductBasis(
                interaction_irreps, hidden_out, self.correlation[0], num_elements,
                use_sc="Residual" in interaction_first))
            self.readouts.append(LinearReadout(hidden_out))
            for i in range(num_interactions - 1):
                last = i == num_interactions - 2
                hidden_out = Irreps(str(hid[0])) if last else hid
                self.interactions.append(INTERACTIONS[interaction](
                    self.node_attr_irreps, hid, self.irreps_sh, edge_feats_irreps,
                    interaction_irreps, hidden_out, avg_num_neighbors, radial_MLP))
                self.products.append(EquivariantProductBasis(
                    interaction_irreps, hidden_out, self.correlation[i + 1], num_elements, use_sc=True))
                self.readouts.append(NonLinearReadout(hidden_out, MLP_irreps, gate_fn) if last
                                     else LinearReadout(hid))
        self.use_fast = "auto"
        #: in evaluation, run the fused path's edge work in receiver chunks of at most this many
        #: edges under activation checkpointing (``None``: one pass over all edges)
        self.edge_chunk = None
        self.__dict__["_fast_cache"] = None

    # --- fast-path selection -----------------------------------------------------
    #: ``"auto"``: the fused path on any CUDA input the architecture allows (measured faster from
    #: the smallest benchmark batches on)
    AUTO_POLICY = AutoPolicy()

    def set_use_fast(self, use_fast) -> "MACE":
        self.use_fast = resolve_use_fast(use_fast)
        return self

    def fast_eligible(self) -> bool:
        """Whether the fused path covers this architecture (scalar hidden features, l <= 3)."""
        if len(self.interactions) == 0 or self.max_ell > 3 or self.distance_transform is not None:
            return False
        if self.edge_feat.radial_type != "bessel" or self.pair_repulsion:
            return False
        if any(c > 3 for c in self.correlation[:len(self.interactions)]):
            return False
        for blk in self.interactions:
            if blk.density or blk.node_feats_irreps.lmax > 0 or len(blk.conv_tp_weights) != 4:
                return False
        for prod in self.products:
            if prod.symmetric_contractions.irreps_out.lmax > 0:
                return False
        return True

    def _fast_active(self, like: Tensor) -> bool:
        covered = self.fast_eligible() and like.dtype in (torch.float32, torch.float64)
        if self.use_fast is True:
            return covered          # the PyTorch twin of the fused path also runs on the CPU
        return choose(self.use_fast, covered, self.AUTO_POLICY, like.device, like.dtype, int(like.shape[0]))

    # --- energies ----------------------------------------------------------------
    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor,
                             plan=None) -> Tuple[Tensor, Tensor]:
        if self._fast_active(edge_vec):
            from .mace_fast import fast_node_features_energy
            return fast_node_features_energy(self, atomic_numbers, edge_index, edge_vec, plan)
        node_attrs = self.node_attr(atomic_numbers)
        e0 = self.atom_ref(atomic_numbers).squeeze(-1)
        n = atomic_numbers.shape[0]
        lengths = torch.linalg.norm(edge_vec, dim=-1)
        edge_sh = self.edge_feat.sph(edge_vec)
        r_basis = lengths if self.distance_transform is None else self.distance_transform(
            lengths, atomic_numbers, edge_index)
        edge_radial = self.edge_feat.rbf(r_basis) * self.edge_feat.envelope(lengths)[:, None]
        inter = torch.zeros_like(e0)
        if self.pair_repulsion:
            inter = inter + self.pair_repulsion_fn(lengths[:, None], atomic_numbers, edge_index, n)
        node_feats = self.node_embedding(node_attrs)
        feats_list = []
        for t, (interaction, product, readout) in enumerate(zip(self.interactions, self.products,
                                                                 self.readouts)):
            if t > 0:
                node_feats = refresh_ghosts(node_feats)
            node_feats, sc = interaction(node_attrs, node_feats, edge_sh, edge_radial, edge_index)
            node_feats = product(node_feats, sc, node_attrs)
            inter = inter + readout(node_feats).squeeze(-1)
            feats_list.append(node_feats[:, :self._n_scalar_features])
        if not feats_list:
            feats_list.append(node_feats)
        return torch.cat(feats_list, dim=-1), e0 + self.scale_shift(inter)

    def node_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor) -> Tensor:
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def receptive_field(self) -> float:
        return len(self.interactions) * float(self.cutoff)

    def forward(self, data: AtomicGraph) -> dict:
        edge_vec = data.edge_vectors()
        plan = None
        if data.edge_order == "dst" and self._fast_active(edge_vec):
            from ..ops.mace_ops import EdgePlan
            plan = (EdgePlan.from_packed(data.edge_index, data.num_nodes, data.edge_plan)
                    if data.edge_plan is not None else
                    EdgePlan.build(data.edge_index, data.num_nodes, assume_dst_sorted=True))
        feats, node_energy = self.node_features_energy(data.atomic_numbers, data.edge_index,
                                                       edge_vec, plan)
        return {"node_energy": node_energy, "energy": self.aggregate_energy(node_energy, data),
                "node_features": feats}

    @classmethod
    def from_config(cls, cfg) -> "MACE":
        from ..config.coerce import coerce_per_species, coerce_species
        extra = dict(cfg.extra or {})
        species = coerce_species(extra.get("species"), default=[1, 6, 8])
        ae = coerce_per_species(extra.get("atomic_energies"), species, "atomic_energies")
        radial_MLP = extra.get("radial_MLP")
        if isinstance(radial_MLP, str):
            radial_MLP = ast.literal_eval(radial_MLP)
        return cls(species=species, cutoff=cfg.cutoff, max_ell=extra.get("max_ell", 3),
                   max_L=extra.get("max_L", 0), num_channels=cfg.n_features, n_rbf=cfg.n_rbf,
                   num_interactions=cfg.n_interactions, correlation=extra.get("correlation", 3),
                   MLP_irreps=extra.get("MLP_irreps", "16x0e"), radial_MLP=radial_MLP,
                   interaction=extra.get("interaction", "RealAgnosticResidualInteractionBlock"),
                   interaction_first=extra.get("interaction_first",
                                               "RealAgnosticResidualInteractionBlock"),
                   gate=extra.get("gate", "silu"),
                   avg_num_neighbors=extra.get("avg_num_neighbors", 1.0),
                   hidden_irreps=extra.get("hidden_irreps"),
                   num_cutoff_basis=extra.get("num_polynomial_cutoff", 5),
                   radial_type=extra.get("radial_type", "bessel"),
                   distance_transform=extra.get("distance_transform", "None"),
                   pair_repulsion=extra.get("pair_repulsion", False), atomic_energies=ae,
                   scale=float(extra.get("scale", 1.0)), shift=float(extra.get("shift", 0.0)),
                   rbf_prefactor=extra.get("rbf_prefactor"))


def _hidden(num_channels: int, max_L: int) -> Irreps:
    return hidden_irreps(num_channels, max_L)


def hidden_irreps_of(mul: int, lmax: int) -> Irreps:
    return hidden_irreps(mul, lmax)
