"""DimeNet (Gasteiger et al., ICLR 2020) and DimeNet++ (2020): directional message passing on
edge messages ``m_ji`` with triplets ``k -> j -> i`` (the reverse edge excluded), Bessel radial
and spherical Fourier-Bessel bases under a polynomial envelope, bilinear (DimeNet) or
down/up-projected Hadamard (DimeNet++) triplet interactions, residual stacks and per-block
output heads summed into atomic energies. Options, initialisation forms and parameter names
follow the reference (``src/xnn/gnn/models/dimenet.py``) so that weights transplant.
"""
from __future__ import annotations

import math
from typing import List, Optional, Tuple

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..featurizers.spherical_bessel import SphericalBesselBasis
from ..nn.blocks import make_activation
from ..nn.cutoff import PolynomialCutoff
from ..nn.radial import BesselRBF
from ..ops.scatter import scatter_sum
from .base import InteratomicPotential
from .registry import register_model

_MAX_Z = 100


def glorot_orthogonal_(w: Tensor, scale: float = 2.0) -> Tensor:
    """An orthogonal matrix rescaled to the Glorot variance ``scale / (fan_in + fan_out)``."""
    with torch.no_grad():
        nn.init.orthogonal_(w)
        w.mul_(math.sqrt(scale / ((w.shape[0] + w.shape[1]) * w.var())))
    return w


def _dense(n_in: int, n_out: int, bias: bool = True, init: str = "glorot_orthogonal") -> nn.Linear:
    lin = nn.Linear(n_in, n_out, bias=bias)
    if init == "zeros":
        nn.init.zeros_(lin.weight)
    elif init == "glorot_orthogonal":
        glorot_orthogonal_(lin.weight)
    else:
        raise ValueError(f"init must be 'zeros' or 'glorot_orthogonal', got {init!r}")
    if bias:
        nn.init.zeros_(lin.bias)
    return lin


def directed_triplets(edge_index: Tensor, edge_vec: Tensor, num_nodes: int) -> Tuple[Tensor, Tensor]:
    """``(kj, ji)``: for every edge ``j -> i`` each edge ``k -> j`` into its source, except the
    reverse of ``j -> i`` itself (same atoms, opposite vector)."""
    src, dst = edge_index[0], edge_index[1]
    counts = torch.bincount(dst, minlength=num_nodes)
    order = torch.argsort(dst, stable=True)
    starts = torch.cumsum(counts, 0) - counts
    n_in = counts[src]
    ji = torch.repeat_interleave(torch.arange(src.shape[0], device=src.device), n_in)
    local = torch.arange(ji.shape[0], device=src.device) - torch.repeat_interleave(torch.cumsum(n_in, 0) - n_in, n_in)
    kj = order[starts[src[ji]] + local]
    vec = edge_vec.detach()
    keep = ~((src[kj] == dst[ji]) & (vec[kj] + vec[ji] == 0).all(-1))
    return kj[keep], ji[keep]


class _Residual(nn.Module):
    def __init__(self, n: int, act: nn.Module):
        super().__init__()
        self.lin1, self.lin2, self.act = _dense(n, n), _dense(n, n), act

    def forward(self, x: Tensor) -> Tensor:
        return x + self.act(self.lin2(self.act(self.lin1(x))))


class _Embedding(nn.Module):
    def __init__(self, n: int, n_rbf: int, act: nn.Module):
        super().__init__()
        self.embedding = nn.Embedding(_MAX_Z, n)
        nn.init.uniform_(self.embedding.weight, -math.sqrt(3.0), math.sqrt(3.0))
        self.lin_rbf, self.lin, self.act = _dense(n_rbf, n), _dense(3 * n, n), act

    def forward(self, z: Tensor, edge_index: Tensor, rbf: Tensor) -> Tensor:
        h = self.embedding(z)
        x = torch.cat([h.index_select(0, edge_index[0]), h.index_select(0, edge_index[1]), self.act(self.lin_rbf(rbf))], -1)
        return self.act(self.lin(x))


class _Skip(nn.Module):
    def _finish(self, x: Tensor, m: Tensor) -> Tensor:
        for blk in self.before_skip:
            x = blk(x)
        m = m + self.act(self.lin_skip(x))
        for blk in self.after_skip:
            m = blk(m)
        return m


class _Interaction(_Skip):
    def __init__(self, n: int, n_rbf: int, n_sbf: int, n_bilinear: int, n_before: int, n_after: int, act: nn.Module,
                 radial_gate: str = "kj"):
        super().__init__()
        self.lin_rbf = _dense(n_rbf, n, bias=False)
        self.lin_sbf = _dense(n_sbf, n_bilinear, bias=False)
        self.lin_ji, self.lin_kj = _dense(n, n), _dense(n, n)
        self.bilinear = nn.Parameter(torch.empty(n_bilinear, n, n))
        nn.init.normal_(self.bilinear, 0.0, 2.0 / n)
        self.before_skip = nn.ModuleList([_Residual(n, act) for _ in range(n_before)])
        self.lin_skip = _dense(n, n)
        self.after_skip = nn.ModuleList([_Residual(n, act) for _ in range(n_after)])
        self.act, self.radial_gate = act, radial_gate

    def forward(self, m: Tensor, rbf: Tensor, sbf: Tensor, kj: Tensor, ji: Tensor) -> Tensor:
        x_ji, x_kj = self.act(self.lin_ji(m)), self.act(self.lin_kj(m))
        gate, s = self.lin_rbf(rbf), self.lin_sbf(sbf)
        nb, nf, ng = self.bilinear.shape
        if self.radial_gate == "ji":
            t = x_kj.index_select(0, kj) * gate.index_select(0, ji)
            msg = torch.einsum("tb,tf,bfg->tg", s, t, self.bilinear)
        else:
            proj = (x_kj * gate) @ self.bilinear.permute(1, 0, 2).reshape(nf, nb * ng)
            msg = torch.bmm(s.unsqueeze(1), proj.index_select(0, kj).view(-1, nb, ng)).squeeze(1)
        return self._finish(x_ji + scatter_sum(msg, ji, m.shape[0]), m)


class _InteractionPP(_Skip):
    def __init__(self, n: int, n_rbf: int, n_sbf: int, n_triplet: int, n_basis: int, n_before: int, n_after: int,
                 act: nn.Module, radial_gate: str = "kj"):
        super().__init__()
        self.lin_rbf1, self.lin_rbf2 = _dense(n_rbf, n_basis, bias=False), _dense(n_basis, n, bias=False)
        self.lin_sbf1, self.lin_sbf2 = _dense(n_sbf, n_basis, bias=False), _dense(n_basis, n_triplet, bias=False)
        self.lin_ji, self.lin_kj = _dense(n, n), _dense(n, n)
        self.lin_down, self.lin_up = _dense(n, n_triplet, bias=False), _dense(n_triplet, n, bias=False)
        self.before_skip = nn.ModuleList([_Residual(n, act) for _ in range(n_before)])
        self.lin_skip = _dense(n, n)
        self.after_skip = nn.ModuleList([_Residual(n, act) for _ in range(n_after)])
        self.act, self.radial_gate = act, radial_gate

    def forward(self, m: Tensor, rbf: Tensor, sbf: Tensor, kj: Tensor, ji: Tensor) -> Tensor:
        x_ji, x_kj = self.act(self.lin_ji(m)), self.act(self.lin_kj(m))
        gate = self.lin_rbf2(self.lin_rbf1(rbf))
        if self.radial_gate == "ji":
            x_kj = self.act(self.lin_down(x_kj.index_select(0, kj) * gate.index_select(0, ji)))
        else:
            x_kj = self.act(self.lin_down(x_kj * gate)).index_select(0, kj)
        agg = self.act(self.lin_up(scatter_sum(x_kj * self.lin_sbf2(self.lin_sbf1(sbf)), ji, m.shape[0])))
        return self._finish(x_ji + agg, m)


class _Output(nn.Module):
    def __init__(self, n: int, n_rbf: int, n_out: Optional[int], n_layers: int, act: nn.Module, output_init: str):
        super().__init__()
        self.lin_rbf = _dense(n_rbf, n, bias=False)
        self.up = None if n_out is None else _dense(n, n_out, bias=False)
        width = n if n_out is None else n_out
        self.dense = nn.ModuleList([_dense(width, width) for _ in range(n_layers)])
        self.final = _dense(width, 1, bias=False, init=output_init)
        self.act = act

    def forward(self, m: Tensor, rbf: Tensor, dst: Tensor, num_nodes: int):
        h = scatter_sum(m * self.lin_rbf(rbf), dst, num_nodes)
        if self.up is not None:
            h = self.up(h)
        for lin in self.dense:
            h = self.act(lin(h))
        return h, self.final(h).squeeze(-1)


@register_model("dimenet")
class DimeNet(InteratomicPotential):
    head_modules = ("outputs", "atom_ref")

    def __init__(self, n_features: int = 128, n_interactions: int = 6, n_rbf: int = 6, n_spherical: int = 7,
                 cutoff: float = 5.0, n_bilinear: int = 8, n_output_features: Optional[int] = None, p: int = 6,
                 n_before_skip: int = 1, n_after_skip: int = 2, n_output_layers: int = 3, activation="silu",
                 output_init: str = "glorot_orthogonal", trainable_rbf: bool = True, radial_gate: str = "kj",
                 reference_basis: bool = False, species=None, atomic_energies=None):
        super().__init__()
        act = make_activation(activation)
        self._init_trunk(n_features, n_rbf, n_spherical, cutoff, n_output_features, p, n_interactions,
                         n_output_layers, act, output_init, trainable_rbf, radial_gate, reference_basis, species,
                         atomic_energies)
        self.interactions = nn.ModuleList([_Interaction(n_features, n_rbf, self.n_sbf, n_bilinear, n_before_skip,
                                                        n_after_skip, act, radial_gate) for _ in range(n_interactions)])

    def _init_trunk(self, n_features, n_rbf, n_spherical, cutoff, n_output_features, p, n_interactions,
                    n_output_layers, act, output_init, trainable_rbf, radial_gate, reference_basis, species,
                    atomic_energies) -> None:
        if output_init not in ("zeros", "glorot_orthogonal"):
            raise ValueError(f"output_init must be 'zeros' or 'glorot_orthogonal', got {output_init!r}")
        if radial_gate not in ("kj", "ji"):
            raise ValueError(f"radial_gate must be 'kj' or 'ji', got {radial_gate!r}")
        self.cutoff = float(cutoff)
        self.radial_gate, self.reference_basis = radial_gate, reference_basis
        if species is not None:
            self.species = [int(z) for z in species]
        self.node_feature_dim = n_features if n_output_features is None else n_output_features
        self.rbf = BesselRBF(n_rbf, cutoff, trainable=trainable_rbf)
        self.sbf = SphericalBesselBasis(n_spherical, n_rbf, cutoff)
        self.n_sbf = self.sbf.output_dim
        self.envelope = PolynomialCutoff(cutoff, p)
        self.embedding = _Embedding(n_features, n_rbf, act)
        self.outputs = nn.ModuleList([_Output(n_features, n_rbf, n_output_features, n_output_layers, act, output_init)
                                      for _ in range(n_interactions + 1)])
        self.atom_ref = nn.Embedding(_MAX_Z, 1)
        nn.init.zeros_(self.atom_ref.weight)
        if atomic_energies is not None:
            if species is None:
                raise ValueError("species is required to map atomic_energies")
            self.set_atomic_energies(species, atomic_energies)

    def set_atomic_energies(self, species, values) -> None:
        ae = torch.as_tensor(values, dtype=self.atom_ref.weight.dtype)
        with torch.no_grad():
            self.atom_ref.weight[torch.tensor(list(species)), 0] = ae

    def receptive_field(self) -> float:
        return (len(self.interactions) + 1) * self.cutoff

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        kj, ji = directed_triplets(edge_index, edge_vec, atomic_numbers.shape[0])
        return self._features_energy(atomic_numbers, edge_index, edge_vec, kj, ji)

    def _features_energy(self, z, edge_index, edge_vec, kj, ji):
        n = z.shape[0]
        dst = edge_index[1]
        r = torch.linalg.norm(edge_vec, dim=-1)
        env = self.envelope(r)
        rbf = self.rbf(r) * env[:, None]
        cos_a = -(edge_vec.index_select(0, kj) * edge_vec.index_select(0, ji)).sum(-1) / (r[kj] * r[ji])
        cos_a = cos_a.clamp(-1.0, 1.0)
        env_sbf = env * (self.cutoff / r) if self.reference_basis else env
        radial = self.sbf.radial(r) * env_sbf[:, None, None]
        sbf = (radial.index_select(0, kj) * self.sbf.angular(cos_a)[:, :, None]).reshape(kj.shape[0], self.n_sbf)
        m = self.embedding(z, edge_index, rbf)
        messages: List[Tensor] = [m]
        for blk in self.interactions:
            m = blk(m, rbf, sbf, kj, ji)
            messages.append(m)
        feats = torch.zeros(n, self.node_feature_dim, dtype=m.dtype, device=m.device)
        node = self.atom_ref(z).squeeze(-1)
        for i, out in enumerate(self.outputs):
            h, t = out(messages[i], rbf, dst, n)
            feats, node = feats + h, node + t
        return feats, node

    def node_energy(self, atomic_numbers, edge_index, edge_vec):
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> dict:
        f, e = self.node_features_energy(data.atomic_numbers, data.edge_index, data.edge_vectors())
        return {"node_energy": e, "energy": self.aggregate_energy(e, data), "node_features": f}

    @staticmethod
    def _common_options(cfg) -> dict:
        e = dict(cfg.extra or {})
        p = e.get("p")
        if p is None:
            p = int(e.get("envelope_exponent", 5)) + 1
        n_out = e.get("n_output_features")
        return dict(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf, cutoff=cfg.cutoff,
                    n_spherical=int(e.get("n_spherical", 7)), n_output_features=None if n_out is None else int(n_out),
                    p=int(p), n_before_skip=int(e.get("n_before_skip", 1)), n_after_skip=int(e.get("n_after_skip", 2)),
                    n_output_layers=int(e.get("n_output_layers", 3)), activation=e.get("activation", "silu"),
                    output_init=e.get("output_init", "glorot_orthogonal"),
                    trainable_rbf=bool(e.get("trainable_rbf", True)), radial_gate=str(e.get("radial_gate", "kj")),
                    reference_basis=bool(e.get("reference_basis", False)), species=e.get("species"),
                    atomic_energies=e.get("atomic_energies"))

    @classmethod
    def from_config(cls, cfg) -> "DimeNet":
        return cls(n_bilinear=int(dict(cfg.extra or {}).get("n_bilinear", 8)), **cls._common_options(cfg))


@register_model("dimenet++")
class DimeNetPP(DimeNet):
    def __init__(self, n_features: int = 128, n_interactions: int = 4, n_rbf: int = 6, n_spherical: int = 7,
                 cutoff: float = 5.0, n_triplet_features: int = 64, n_basis_features: int = 8,
                 n_output_features: int = 256, p: int = 6, n_before_skip: int = 1, n_after_skip: int = 2,
                 n_output_layers: int = 3, activation="silu", output_init: str = "glorot_orthogonal",
                 trainable_rbf: bool = True, radial_gate: str = "kj", reference_basis: bool = False, species=None,
                 atomic_energies=None):
        InteratomicPotential.__init__(self)
        act = make_activation(activation)
        self._init_trunk(n_features, n_rbf, n_spherical, cutoff, n_output_features, p, n_interactions,
                         n_output_layers, act, output_init, trainable_rbf, radial_gate, reference_basis, species,
                         atomic_energies)
        self.interactions = nn.ModuleList([_InteractionPP(n_features, n_rbf, self.n_sbf, n_triplet_features,
                                                          n_basis_features, n_before_skip, n_after_skip, act,
                                                          radial_gate) for _ in range(n_interactions)])

    @classmethod
    def from_config(cls, cfg) -> "DimeNetPP":
        e = dict(cfg.extra or {})
        opts = cls._common_options(cfg)
        if opts["n_output_features"] is None:
            opts["n_output_features"] = 256
        return cls(n_triplet_features=int(e.get("n_triplet_features", 64)),
                   n_basis_features=int(e.get("n_basis_features", 8)), **opts)
