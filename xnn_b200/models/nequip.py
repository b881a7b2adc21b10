"""NequIP (Batzner et al. 2022): E(3)-equivariant interatomic potential with gated nonlinearities.

Structure and state-dict names follow the reference (``src/xnn/gnn/models/nequip.py:124-848``):
a one-hot ``chemical_embedding``; ``n_layers`` ConvNetLayers, each an InteractionBlock
(``linear_1`` -> radial-MLP-weighted ``uvu`` tensor product with the spherical harmonics of
``-r_ij`` -> sum over neighbours / sqrt(avg_num_neighbors) -> ``linear_2`` + species
self-connection ``sc``) followed by a gate (scalars activated, higher irreps multiplied by
activated scalar gates); then ``conv_to_output_hidden`` and ``output_hidden_to_scalar`` and a
per-species scale and shift. Bessel frequencies are trainable with prefactor ``2 / r_max``.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from ..data import AtomicGraph
from ..nn import BesselRBF, PolynomialCutoff
from ..o3 import (FullyConnectedNet, FullyConnectedTensorProduct, Irrep, Irreps, Linear, TensorProduct,
                  normalize2mom, spherical_harmonics)
from ..ops.scatter import scatter_sum
from .base import GNNPotential
from .mace import ScalarActivation
from .mace_blocks import tp_out_irreps_with_instructions
from .registry import register_model


def _ssp(x: Tensor) -> Tensor:
    return F.softplus(x) - math.log(2.0)


ACTS = {"silu": F.silu, "ssp": _ssp, "tanh": torch.tanh, "abs": torch.abs, "None": None, None: None}


def _act_parity(act) -> int:
    """+1 for an even activation, -1 for an odd one, 0 otherwise (checked numerically)."""
    if act is None:
        return 1
    x = torch.linspace(0.1, 3.0, 17, dtype=torch.float64)
    y, ym = act(x), act(-x)
    if torch.allclose(y, ym):
        return 1
    if torch.allclose(y, -ym):
        return -1
    return 0


def nequip_hidden_irreps(num_features: int, l_max: int, parity: bool = True) -> Irreps:
    """``num_features`` channels of every degree, all even irreps first, then the odd ones."""
    out = []
    for p in ([1, -1] if parity else [1]):
        for l in range(l_max + 1):
            out.append((num_features, Irrep(l, p)))
    return Irreps(out)


def tp_path_exists(irreps_in1, irreps_in2, ir_out) -> bool:
    target = Irrep(ir_out)
    for m1, ir1 in Irreps(irreps_in1):
        if m1 == 0:
            continue
        for m2, ir2 in Irreps(irreps_in2):
            if m2 > 0 and target in list(ir1 * ir2):
                return True
    return False


class Gate(nn.Module):
    """Gated nonlinearity on features laid out as ``sort(scalars + gates + gated).simplify()``."""

    def __init__(self, irreps_scalars, act_scalars, irreps_gates, act_gates, irreps_gated):
        super().__init__()
        irreps_scalars = Irreps(irreps_scalars).simplify()
        irreps_gates = Irreps(irreps_gates).simplify()
        irreps_gated = Irreps(irreps_gated).simplify()
        if len(irreps_gates) > 1:
            raise ValueError("expected a single merged gates entry")
        if irreps_gates.num_irreps != irreps_gated.num_irreps:
            raise ValueError("one gate per gated channel is required")
        unsorted = irreps_scalars + irreps_gates + irreps_gated
        srt, perm, _ = unsorted.sort()
        starts = [0]
        for m in srt:
            starts.append(starts[-1] + m.dim)
        self.in_starts = [starts[perm[k]] for k in range(len(unsorted))]
        self.lens = [m.dim for m in unsorted]
        self.n_s, self.n_g = len(irreps_scalars), len(irreps_gates)
        self.scalar_acts = nn.ModuleList([ScalarActivation(Irreps([m]), a)
                                          for m, a in zip(irreps_scalars, act_scalars)])
        self.has_gates = self.n_g > 0
        self.gate_act = ScalarActivation(irreps_gates, act_gates[0] if self.has_gates else None)
        self.gated = list(irreps_gated)
        out = []
        for (mul, ir), act in zip(irreps_scalars, act_scalars):
            if act is None:
                p_out = ir.p
            else:
                pa = _act_parity(act)
                p_out = pa if ir.p == -1 else ir.p
            if p_out == 0:
                raise ValueError(f"an activation on odd scalars must have a parity: {ir}")
            out.append((mul, Irrep(0, p_out)))
        p_gate = irreps_gates[0].ir.p if self.has_gates else 1
        out += [(mul, Irrep(ir.l, ir.p * p_gate)) for mul, ir in irreps_gated]
        self.irreps_out = Irreps(out)
        self.irreps_in = srt.simplify()

    def forward(self, x: Tensor) -> Tensor:
        outs = []
        for i, act in enumerate(self.scalar_acts):
            outs.append(act(x.narrow(-1, self.in_starts[i], self.lens[i])))
        if self.has_gates:
            g = self.gate_act(x.narrow(-1, self.in_starts[self.n_s], self.lens[self.n_s]))
            c = 0
            for j, (mul, ir) in enumerate(self.gated):
                k = self.n_s + self.n_g + j
                piece = x.narrow(-1, self.in_starts[k], self.lens[k]).reshape(*x.shape[:-1], mul, ir.dim)
                piece = piece * g.narrow(-1, c, mul).unsqueeze(-1)
                outs.append(piece.reshape(*x.shape[:-1], mul * ir.dim))
                c += mul
        return torch.cat(outs, -1) if len(outs) > 1 else outs[0]


class InteractionBlock(nn.Module):
    def __init__(self, irreps_in, irreps_out, irreps_node_attr, irreps_edge_attr, n_radial: int,
                 invariant_layers: int = 2, invariant_neurons: int = 64,
                 avg_num_neighbors: Optional[float] = None, use_sc: bool = True,
                 nonlinearity_scalars: Optional[Dict[str, str]] = None):
        super().__init__()
        nl = nonlinearity_scalars or {"e": "silu"}
        self.irreps_in, self.irreps_out = Irreps(irreps_in), Irreps(irreps_out)
        self.avg_num_neighbors = float(avg_num_neighbors) if avg_num_neighbors is not None else None
        self.use_sc = use_sc
        self.linear_1 = Linear(self.irreps_in, self.irreps_in)
        irreps_mid, ins = tp_out_irreps_with_instructions(self.irreps_in, irreps_edge_attr, self.irreps_out,
                                                          sort_instructions=False)
        self.tp = TensorProduct(self.irreps_in, irreps_edge_attr, irreps_mid, ins,
                                shared_weights=False, internal_weights=False)
        self.fc = FullyConnectedNet([n_radial] + invariant_layers * [invariant_neurons] + [self.tp.weight_numel],
                                    ACTS[nl["e"]])
        self.linear_2 = Linear(irreps_mid.simplify(), self.irreps_out)
        if use_sc:
            self.sc = FullyConnectedTensorProduct(self.irreps_in, irreps_node_attr, self.irreps_out)

    def forward(self, x, node_attrs, edge_index, edge_sh, edge_radial):
        x_in = x
        x = self.linear_1(x)
        w = self.fc(edge_radial)
        msg = self.tp(x.index_select(0, edge_index[0]), edge_sh, w)
        out = scatter_sum(msg, edge_index[1], x.shape[0])
        if self.avg_num_neighbors is not None:
            out = out / math.sqrt(self.avg_num_neighbors)
        out = self.linear_2(out)
        if self.use_sc:
            out = out + self.sc(x_in, node_attrs)
        return out


class ConvNetLayer(nn.Module):
    def __init__(self, irreps_in, feature_irreps_hidden, irreps_node_attr, irreps_edge_attr, n_radial: int,
                 resnet: bool = False, nonlinearity_scalars=None, nonlinearity_gates=None, **conv_kwargs):
        super().__init__()
        ns = nonlinearity_scalars or {"e": "silu", "o": "tanh"}
        ng = nonlinearity_gates or {"e": "silu", "o": "tanh"}
        irreps_in = Irreps(irreps_in)
        hid = Irreps(feature_irreps_hidden)
        acts_s = {1: ACTS[ns["e"]], -1: ACTS[ns["o"]]}
        acts_g = {1: ACTS[ng["e"]], -1: ACTS[ng["o"]]}
        scal = Irreps([(m, ir) for m, ir in hid if ir.l == 0 and tp_path_exists(irreps_in, irreps_edge_attr, ir)])
        gated = Irreps([(m, ir) for m, ir in hid if ir.l > 0 and tp_path_exists(irreps_in, irreps_edge_attr, ir)])
        ir_gate = "0e" if tp_path_exists(irreps_in, irreps_edge_attr, "0e") else "0o"
        n_gated = sum(m for m, _ in gated)
        gates = Irreps([(n_gated, ir_gate)]) if n_gated > 0 else Irreps([])
        self.equivariant_nonlin = Gate(scal, [acts_s[ir.p] for _, ir in scal], gates,
                                       [acts_g[Irrep(ir_gate).p]] if n_gated > 0 else [], gated)
        self.conv = InteractionBlock(irreps_in, self.equivariant_nonlin.irreps_in.simplify(), irreps_node_attr,
                                     irreps_edge_attr, n_radial, nonlinearity_scalars=ns, **conv_kwargs)
        self.irreps_out = self.equivariant_nonlin.irreps_out
        self.resnet = bool(resnet) and self.irreps_out == irreps_in

    def forward(self, x, node_attrs, edge_index, edge_sh, edge_radial):
        old = x
        x = self.conv(x, node_attrs, edge_index, edge_sh, edge_radial)
        x = self.equivariant_nonlin(x)
        return old + x if self.resnet else x


@register_model("nequip")
class NequIP(GNNPotential):
    head_modules = ("conv_to_output_hidden", "output_hidden_to_scalar", "atom_ref", "atom_scale")

    def __init__(self, species, cutoff: float = 4.0, l_max: int = 2, parity: bool = True, n_rbf: int = 8,
                 n_layers: int = 3, num_features: int = 32, invariant_layers: int = 2,
                 invariant_neurons: int = 64, avg_num_neighbors: Optional[float] = None, use_sc: bool = True,
                 resnet: bool = False, nonlinearity_scalars=None, nonlinearity_gates=None,
                 num_polynomial_cutoff: int = 6, trainable_rbf: bool = True,
                 conv_to_output_hidden: Optional[int] = None, atomic_energies=None, atomic_scales=None):
        if n_layers < 0:
            raise ValueError("n_layers (num_layers) must be >= 0")
        super().__init__(species, cutoff)
        self.l_max = l_max
        self.node_attr_irreps = Irreps([(len(self.species), "0e")])
        self.irreps_sh = Irreps.spherical_harmonics(l_max, p=-1 if parity else 1)
        # the radial basis sits in ``edge_feat`` as in the reference's shared edge featurizer
        # (``edge_feat.rbf.freqs`` in the state dict)
        self.edge_feat = nn.Module()
        self.edge_feat.rbf = BesselRBF(n_rbf, cutoff, trainable=trainable_rbf, prefactor=2.0 / cutoff)
        self.envelope = PolynomialCutoff(cutoff, p=num_polynomial_cutoff)
        ns = nonlinearity_scalars or {"e": "silu", "o": "tanh"}
        ng = nonlinearity_gates or {"e": "silu", "o": "tanh"}
        hidden_irreps = nequip_hidden_irreps(num_features, l_max, parity)
        irreps = Irreps([(num_features, "0e")])
        self.chemical_embedding = Linear(self.node_attr_irreps, irreps)
        self.layers = nn.ModuleList()
        for _ in range(n_layers):
            layer = ConvNetLayer(irreps, hidden_irreps, self.node_attr_irreps, self.irreps_sh, n_rbf,
                                 resnet=resnet, nonlinearity_scalars=ns, nonlinearity_gates=ng,
                                 invariant_layers=invariant_layers, invariant_neurons=invariant_neurons,
                                 avg_num_neighbors=avg_num_neighbors, use_sc=use_sc)
            self.layers.append(layer)
            irreps = layer.irreps_out
        hidden = conv_to_output_hidden if conv_to_output_hidden is not None else max(1, num_features // 2)
        irreps_out_hidden = Irreps([(hidden, "0e")])
        self.conv_to_output_hidden = Linear(irreps, irreps_out_hidden)
        self.node_feature_dim = irreps_out_hidden.dim
        self.output_hidden_to_scalar = Linear(irreps_out_hidden, "1x0e")
        self.register_buffer("atom_scale", torch.ones(200))
        if atomic_scales is not None:
            sc = torch.as_tensor(atomic_scales, dtype=self.atom_scale.dtype)
            if sc.numel() != len(self.species):
                raise ValueError(f"got {sc.numel()} atomic scales for {len(self.species)} species")
            self.atom_scale[torch.tensor(self.species)] = sc
        if atomic_energies is not None:
            self.set_atomic_energies(atomic_energies)

    @property
    def rbf(self) -> nn.Module:
        return self.edge_feat.rbf

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        old = prefix + "rbf.freqs"          # the earlier top-level name
        if old in state_dict:
            state_dict[prefix + "edge_feat.rbf.freqs"] = state_dict.pop(old)
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        node_attrs = self.node_attr(atomic_numbers)
        vec = -edge_vec                       # NequIP evaluates Y_l on r_j - r_i
        r = torch.linalg.norm(vec, dim=-1)
        edge_sh = spherical_harmonics(self.irreps_sh, vec, normalize=True, normalization="component")
        edge_radial = self.rbf(r) * self.envelope(r)[:, None]
        x = self.chemical_embedding(node_attrs)
        for layer in self.layers:
            x = layer(x, node_attrs, edge_index, edge_sh, edge_radial)
        feats = self.conv_to_output_hidden(x)
        eps = self.output_hidden_to_scalar(feats).squeeze(-1)
        return feats, self.atom_scale[atomic_numbers] * eps + self.atom_ref(atomic_numbers).squeeze(-1)

    def node_energy(self, atomic_numbers, edge_index, edge_vec):
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def receptive_field(self) -> float:
        return len(self.layers) * float(self.cutoff)

    def forward(self, data: AtomicGraph) -> dict:
        feats, ne = self.node_features_energy(data.atomic_numbers, data.edge_index, data.edge_vectors())
        return {"node_energy": ne, "energy": self.aggregate_energy(ne, data), "node_features": feats}

    @classmethod
    def from_config(cls, cfg) -> "NequIP":
        from ..config.coerce import coerce_per_species, coerce_species
        extra = dict(cfg.extra or {})
        species = coerce_species(extra.get("species"), default=[1, 6, 8])
        hidden = extra.get("conv_to_output_hidden")
        if isinstance(hidden, str):
            hidden = Irreps(hidden).count("0e")
        avg = extra.get("avg_num_neighbors")
        return cls(species=species, cutoff=cfg.cutoff, l_max=extra.get("l_max", 2),
                   parity=extra.get("parity", True), n_rbf=cfg.n_rbf, n_layers=cfg.n_interactions,
                   num_features=cfg.n_features, invariant_layers=extra.get("invariant_layers", 2),
                   invariant_neurons=extra.get("invariant_neurons", 64),
                   avg_num_neighbors=None if avg is None else float(avg), use_sc=extra.get("use_sc", True),
                   resnet=extra.get("resnet", False),
                   nonlinearity_scalars=extra.get("nonlinearity_scalars"),
                   nonlinearity_gates=extra.get("nonlinearity_gates"),
                   num_polynomial_cutoff=extra.get("num_polynomial_cutoff", 6),
                   trainable_rbf=extra.get("trainable_rbf", True), conv_to_output_hidden=hidden,
                   atomic_energies=coerce_per_species(extra.get("atomic_energies"), species, "atomic_energies"),
                   atomic_scales=coerce_per_species(extra.get("atomic_scales"), species, "atomic_scales"))
