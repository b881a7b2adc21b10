"""Allegro (Musaelian et al., Nat. Commun. 14, 579 (2023)): a strictly local equivariant potential
of pair energies. Every edge carries a scalar latent and a tensor track; each layer weights the
edge's spherical harmonics by an MLP of the latent, sums them over the other edges of the centre
(the environment), couples the tensor track with it in a per-channel ("uuu") weightless tensor
product, mixes same-irrep outputs with a strided linear map and feeds the new scalars back into the
latent (cumulative-softmax residual). ``E_i = sigma_Z sum_j E_ij + mu_Z``.

Conventions (upstream v0.3, as in the reference ``src/xnn/gnn/models/allegro.py``): trainable
Bessel basis with prefactor ``r_c / pi``, SH on ``r_j - r_i``, environment normalised by
``1/sqrt(avg_num_neighbors - 1)`` with the edge removed from its own environment, edge energies by
``1/sqrt(avg_num_neighbors)``, Wigner-3j blocks scaled by ``sqrt(2 l_out + 1)``, strided linear
normalised by ``1/sqrt(mul n_paths)`` with the upstream flat weight layout, forward growth and
backward pruning of the tensor irreps. Parameter names follow the reference so state dicts
transplant.
"""
from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn import PolynomialCutoff
from ..nn.radial import BesselRBF
from ..o3 import FullyConnectedNet, Irrep, Irreps, spherical_harmonics, wigner_3j
from ..ops.scatter import gather_rows, scatter_sum
from .base import GNNPotential
from .nequip import tp_path_exists
from .registry import register_model


class ChannelWeighter(nn.Module):
    """Per channel ``u`` and irrep entry ``r`` one weight multiplying all ``2l+1`` components:
    ``(E, dim) x (E, mul * n_irreps) -> (E, mul, dim)``, times ``alpha``."""

    def __init__(self, irreps, mul_out: int, alpha: float = 1.0):
        super().__init__()
        irreps = Irreps(irreps)
        self.n_irreps, self.mul_out = len(irreps), int(mul_out)
        self.weight_numel = self.n_irreps * self.mul_out
        which = torch.arange(self.n_irreps).repeat_interleave(torch.tensor([ir.dim for _, ir in irreps]))
        self.register_buffer("_which_irrep", which, persistent=False)
        self.alpha = float(alpha)

    def forward(self, attr: Tensor, weights: Tensor, prescaled: bool = False) -> Tensor:
        w = weights.reshape(-1, self.mul_out, self.n_irreps)[:, :, self._which_irrep]
        if self.alpha != 1.0 and not prescaled:
            w = w * self.alpha
        return attr.unsqueeze(-2) * w


class Contracter(nn.Module):
    """Per-channel weightless tensor product ``(E, mul, d1) x (E, mul, d2) -> (E, mul, d_out)``
    through a block Wigner-3j tensor (one block per instruction, scaled by ``sqrt(2 l_out + 1)``)."""

    def __init__(self, irs1: List[Irrep], irs2: List[Irrep], instructions: List[Tuple[int, int, Irrep]]):
        super().__init__()
        off1, off2 = [0], [0]
        for ir in irs1:
            off1.append(off1[-1] + ir.dim)
        for ir in irs2:
            off2.append(off2[-1] + ir.dim)
        self.dim_out = sum(ir.dim for _, _, ir in instructions)
        w = torch.zeros(self.dim_out, off1[-1], off2[-1], dtype=torch.float64)
        k = 0
        for i1, i2, ir in instructions:
            l1, l2 = irs1[i1].l, irs2[i2].l
            w[k:k + ir.dim, off1[i1]:off1[i1] + 2 * l1 + 1, off2[i2]:off2[i2] + 2 * l2 + 1] = \
                wigner_3j(ir.l, l1, l2, dtype=torch.float64) * math.sqrt(2 * ir.l + 1)
            k += ir.dim
        self.register_buffer("_w3j", w.to(torch.get_default_dtype()))
        # a block tensor with entries only at i == j (all-scalar layers) is an inner product
        self.diagonal = off1[-1] == off2[-1] and bool((w - torch.diag_embed(torch.diagonal(w, dim1=1, dim2=2)) == 0).all())

    def forward(self, x1: Tensor, x2: Tensor) -> Tensor:
        z, u, d1 = x1.shape
        d2 = x2.shape[2]
        if self.diagonal:
            diag = torch.diagonal(self._w3j, dim1=1, dim2=2)            # (d_out, d)
            return (x1 * x2).reshape(z * u, d1).mm(diag.t()).reshape(z, u, -1)
        outer = (x1.unsqueeze(3) * x2.unsqueeze(2)).reshape(z * u, d1 * d2)
        return outer.mm(self._w3j.reshape(self.dim_out, d1 * d2).t()).reshape(z, u, -1)


class StridedLinear(nn.Module):
    """Mixes the consecutive same-irrep entries of the tensor-product output into each output irrep,
    ``1/sqrt(mul n)`` normalised; the flat weight ``w`` uses the upstream layout (output order, each
    group ``[v, u, n]``)."""

    def __init__(self, irs_in: List[Irrep], irs_out: List[Irrep], mul: int):
        super().__init__()
        self.mul = int(mul)
        off = [0]
        for ir in irs_in:
            off.append(off[-1] + ir.dim)
        self.groups = []
        for ir_out in irs_out:
            idx = [i for i, ir in enumerate(irs_in) if ir == ir_out]
            if idx != list(range(idx[0], idx[-1] + 1)):
                raise ValueError("inputs of one output irrep must be consecutive")
            self.groups.append((off[idx[0]], off[idx[-1] + 1], len(idx), ir_out.dim, 1.0 / math.sqrt(mul * len(idx))))
        total = sum(mul * n * mul for _, _, n, _, _ in self.groups)
        self.w = nn.Parameter(torch.empty(total).uniform_(-math.sqrt(3.0), math.sqrt(3.0)))

    def forward(self, x: Tensor) -> Tensor:
        E, outs, at = x.shape[0], [], 0
        for start, stop, n, d, norm in self.groups:
            piece = x[:, :, start:stop].reshape(E, self.mul * n, d)
            wg = self.w[at:at + self.mul * self.mul * n].reshape(self.mul, self.mul * n) * norm
            at += self.mul * self.mul * n
            rows = piece.transpose(1, 2).reshape(E * d, self.mul * n)
            outs.append(rows.mm(wg.t()).reshape(E, d, self.mul).transpose(1, 2))
        return torch.cat(outs, -1)


def _mlp(net: FullyConnectedNet, x: Tensor, scale: Optional[Tensor] = None) -> Tensor:
    y = net(x)
    return y if scale is None else y * scale


@register_model("allegro")
class Allegro(GNNPotential):
    def __init__(self, species: List[int], cutoff: float = 6.0, l_max: int = 1, parity: str = "o3_full",
                 n_rbf: int = 8, num_layers: int = 2, num_tensor_features: int = 32,
                 two_body_latent: Optional[List[int]] = None, latent: Optional[List[int]] = None,
                 env_embed: Optional[List[int]] = None, edge_eng: Optional[List[int]] = None,
                 initial_scalar_embedding_dim: Optional[int] = None, avg_num_neighbors: Optional[float] = None,
                 latent_resnet: bool = True, num_polynomial_cutoff: int = 6, trainable_rbf: bool = True,
                 atomic_energies=None, atomic_scales=None):
        if num_layers < 1:
            raise ValueError("num_layers must be >= 1")
        if parity not in ("o3_full", "o3_restricted", "so3"):
            raise ValueError(f"unknown parity setting {parity!r}")
        super().__init__(species, cutoff)
        self.l_max = l_max
        self.edge_feat = nn.Module()
        self.edge_feat.rbf = BesselRBF(n_rbf, cutoff, trainable=trainable_rbf, prefactor=cutoff / math.pi)
        self.edge_feat.envelope = PolynomialCutoff(cutoff, p=num_polynomial_cutoff)
        self.sh_irreps = Irreps.spherical_harmonics(l_max)               # what the SH are evaluated as
        self.irreps_sh = Irreps.spherical_harmonics(l_max, p=1 if parity == "so3" else -1)
        two_body_latent = list(two_body_latent or [32, 64, 128])
        latent, env_embed, edge_eng = list(latent or [128]), list(env_embed or []), list(edge_eng or [32])
        self.num_layers, self.latent_resnet, self.avg_num_neighbors = num_layers, latent_resnet, avg_num_neighbors
        embed_dim = initial_scalar_embedding_dim or two_body_latent[0]
        if embed_dim % 2:
            raise ValueError("initial_scalar_embedding_dim must be even")
        self.type_embeddings = nn.Parameter(torch.randn(2, len(self.species), embed_dim // 2))
        self.basis_embed = FullyConnectedNet([n_rbf, embed_dim], None)
        env_irs = [ir for _, ir in self.irreps_sh]
        allowed = ([Irrep(l, p) for l in range(l_max + 1) for p in (1, -1)] if parity == "o3_full" else list(env_irs))
        tps = [list(env_irs)]
        for layer in range(num_layers):
            want = [Irrep(0, 1)] if layer == num_layers - 1 else allowed
            arg = Irreps([(1, ir) for ir in tps[-1]])
            tps.append([ir for ir in want if tp_path_exists(arg, self.irreps_sh, ir)])
        out = tps[-1]
        pruned = [out]
        for arg in reversed(tps[:-1]):
            out = [a for a in arg if any(any(o in out for o in a * e) for e in env_irs)]
            pruned.append(out)
        tps = list(reversed(pruned))
        self._edge_weighter = ChannelWeighter(self.irreps_sh, num_tensor_features)
        env_alpha = 1.0 / math.sqrt(avg_num_neighbors - 1) if avg_num_neighbors is not None else 1.0
        self._env_weighter = ChannelWeighter(self.irreps_sh, num_tensor_features, alpha=env_alpha)
        self._energy_factor = 1.0 / math.sqrt(avg_num_neighbors) if avg_num_neighbors is not None else 1.0
        self.tps, self.linears, self.latents, self.env_embed_mlps = (nn.ModuleList() for _ in range(4))
        n_scalar_outs = []
        for layer, (arg_irs, out_irs) in enumerate(zip(tps[:-1], tps[1:])):
            instr, full = [], []
            n_scalar = 0
            for ir_out in out_irs:
                for i1, ir1 in enumerate(arg_irs):
                    for i2, ir2 in enumerate(env_irs):
                        if ir_out in ir1 * ir2:
                            n_scalar += ir_out == Irrep(0, 1)
                            instr.append((i1, i2, ir_out))
                            full.append(ir_out)
            n_scalar_outs.append(n_scalar)
            self.tps.append(Contracter(arg_irs, env_irs, instr))
            self.linears.append(StridedLinear(full, out_irs, num_tensor_features))
            width_in = embed_dim if layer == 0 else self.latents[-1].hs[-1] + num_tensor_features * n_scalar_outs[-2]
            self.latents.append(FullyConnectedNet([width_in] + (two_body_latent if layer == 0 else latent), F.silu))
            n_w = self._env_weighter.weight_numel + (self._edge_weighter.weight_numel if layer == 0 else 0)
            self.env_embed_mlps.append(FullyConnectedNet([self.latents[-1].hs[-1]] + env_embed + [n_w],
                                                         F.silu if env_embed else None))
        self._n_scalar_outs = n_scalar_outs
        self._edge_w, self._env_w = self._edge_weighter.weight_numel, self._env_weighter.weight_numel
        self.register_buffer("_env_out_scale", torch.tensor([1.0] * self._edge_w + [env_alpha] * self._env_w),
                             persistent=False)
        self.final_latent = FullyConnectedNet([self.latents[-1].hs[-1] + num_tensor_features * n_scalar_outs[-1]]
                                              + latent, F.silu)
        self.edge_eng = FullyConnectedNet([self.final_latent.hs[-1]] + edge_eng + [1], F.silu)
        self.node_feature_dim = self.final_latent.hs[-1]
        self.register_buffer("_resnet_params", torch.zeros(num_layers + 1))
        self.register_buffer("atom_scale", torch.ones(200))
        if atomic_scales is not None:
            sc = torch.as_tensor(atomic_scales, dtype=self.atom_scale.dtype)
            if sc.numel() != len(self.species):
                raise ValueError(f"got {sc.numel()} atomic scales for {len(self.species)} species")
            self.atom_scale[torch.tensor(self.species)] = sc
        if atomic_energies is not None:
            self.set_atomic_energies(atomic_energies)

    def receptive_field(self):
        return self.cutoff

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        n = atomic_numbers.shape[0]
        center = edge_index[1]
        vec = -edge_vec                                     # Y_l on r_j - r_i
        r = torch.linalg.norm(vec, dim=-1)
        edge_sh = spherical_harmonics(self.sh_irreps, vec, normalize=True, normalization="component")
        radial = self.edge_feat.rbf(r) * self.edge_feat.envelope(r)[:, None]
        types = self.z_to_index[atomic_numbers].clamp(min=0)
        inv = torch.cat([gather_rows(self.type_embeddings[0], types[edge_index[1]]),
                         gather_rows(self.type_embeddings[1], types[edge_index[0]])], -1) * self.basis_embed(radial)
        coeff = (self._resnet_params - self._resnet_params.max()).exp()
        cumsum = coeff.cumsum(0) + 1e-12
        keep, mix = (cumsum[:-1] / cumsum[1:]).sqrt(), (coeff[1:] / cumsum[1:]).sqrt()
        latents, latent_in, feats = None, inv, edge_sh
        for layer, (lat_mlp, env_mlp, tp, lin) in enumerate(zip(self.latents, self.env_embed_mlps, self.tps,
                                                               self.linears)):
            new = lat_mlp(latent_in)
            latents = torch.addcmul(keep[layer - 1] * latents, mix[layer - 1], new) \
                if self.latent_resnet and layer > 0 else new
            scale = self._env_out_scale if layer == 0 else self._env_out_scale[self._edge_w:]
            w = _mlp(env_mlp, latents, scale)
            at = 0
            if layer == 0:
                feats = self._edge_weighter(feats, w[:, :self._edge_w], True)
                at = self._edge_w
            env = self._env_weighter(edge_sh, w[:, at:at + self._env_w], True)
            local = gather_rows(scatter_sum(env, center, n), center) - env
            feats = tp(feats, local)
            scalars = feats[:, :, :self._n_scalar_outs[layer]].reshape(feats.shape[0], -1)
            feats = lin(feats)
            latent_in = torch.cat([latents, scalars], -1)
        new = self.final_latent(latent_in)
        layer = self.num_layers
        latents = torch.addcmul(keep[layer - 1] * latents, mix[layer - 1], new) if self.latent_resnet else new
        e_edge = (self.edge_eng(latents) * self._energy_factor).squeeze(-1)
        eps = scatter_sum(e_edge, center, n)
        return scatter_sum(latents, center, n), (self.atom_scale[atomic_numbers] * eps
                                                 + self.atom_ref(atomic_numbers).squeeze(-1))

    def node_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor) -> Tensor:
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> dict:
        feats, node = self.node_features_energy(data.atomic_numbers, data.edge_index, data.edge_vectors())
        return {"node_energy": node, "energy": self.aggregate_energy(node, data), "node_features": feats}

    @classmethod
    def from_config(cls, cfg) -> "Allegro":
        e = dict(cfg.extra or {})
        keys = ("l_max", "parity", "two_body_latent", "latent", "env_embed", "edge_eng",
                "initial_scalar_embedding_dim", "avg_num_neighbors", "latent_resnet", "num_polynomial_cutoff",
                "trainable_rbf", "atomic_energies", "atomic_scales")
        return cls(species=e.get("species", [1, 6, 8]), cutoff=cfg.cutoff, n_rbf=cfg.n_rbf,
                   num_layers=cfg.n_interactions, num_tensor_features=cfg.n_features,
                   **{k: e[k] for k in keys if k in e})
