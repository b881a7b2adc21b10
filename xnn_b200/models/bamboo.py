"""BAMBOO (Gong et al., Nat. Mach. Intell. 2025): graph equivariant transformer layers with
charge and electronegativity heads, damped Coulomb electrostatics and an optional D3 dispersion
with the CSO damping.

Edges carry ExpNormal radials projected to per-head features; each GET layer gates neighbour
values by an edge-wise attention (``act(q_i . k_j) f_c(r)``), lifts them along the edge direction
into vector messages and updates scalars by ``<v_left, v_right> scale + shift`` (first layer
scalars only, last layer scalars only); charges ``Q_ub tanh(q / Q_ub)`` shifted to the net
charge; ``E = E_nn + chi^2 q + eta^2 q^2 + 1/2 sum_pairs k q_i q_j / r * (r / r_0) / (1 +
softplus_beta((r - r_0) / r_0))`` in kcal/mol. Options, defaults and parameter names follow the
reference (``src/xnn/hybnn/models/bamboo.py``, ``hybnn/models/dispersion.py``).
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.cutoff import CosineCutoff
from ..nn.radial import ExpNormalSmearing
from ..ops.scatter import scatter_sum
from . import d3_legacy
from .base import InteratomicPotential
from .electrostatics import all_pairs
from .registry import register_model

ELE_FACTOR = 332.06349451357806
DEBYE_EA = 0.20819427381112157
HARTREE_KCAL_MOL = 627.5094740631
_ACTS = {"silu": nn.SiLU, "swish": nn.SiLU, "gelu": nn.GELU, "tanh": nn.Tanh, "relu": nn.ReLU}


def _act(a) -> nn.Module:
    if isinstance(a, nn.Module):
        return a
    if str(a).lower() not in _ACTS:
        raise ValueError(f"unknown activation {a!r}; choose from {sorted(_ACTS)}")
    return _ACTS[str(a).lower()]()


def _energy_mlp(n_layers: int, dim: int, act) -> nn.Sequential:
    h = dim // 2
    layers = []
    for i in range(n_layers):
        layers += [nn.Linear(dim if i == 0 else h, h), _act(act)]
    layers.append(nn.Linear(h, 1))
    return nn.Sequential(*layers)


class EdgeMultiheadAttention(nn.Module):
    """Per-edge multi-head gates ``act(q_center . k_neighbor) * envelope`` and the neighbours' values."""

    def __init__(self, dim: int, num_heads: int, act_fn: Optional[nn.Module] = None):
        super().__init__()
        if dim % num_heads:
            raise ValueError(f"dim ({dim}) must be divisible by num_heads ({num_heads})")
        self.dim, self.num_heads, self.dim_per_head = dim, num_heads, dim // num_heads
        self.layer_norm = nn.LayerNorm(dim)
        self.qkv_proj = nn.Linear(dim, 3 * dim)
        self.attn_act = act_fn if act_fn is not None else nn.GELU()

    def forward(self, x: Tensor, center: Tensor, neighbor: Tensor, envelope: Tensor):
        q, k, v = self.qkv_proj(self.layer_norm(x)).unflatten(-1, (self.num_heads, 3, self.dim_per_head)).unbind(-2)
        score = (q.index_select(0, center) * k.index_select(0, neighbor)).sum(-1)
        return v.index_select(0, neighbor), self.attn_act(score) * envelope.unsqueeze(-1)


class GETLayer(nn.Module):
    def __init__(self, dim: int, num_heads: int, attn_act, is_first: bool = False, is_last: bool = False):
        super().__init__()
        self.dim, self.num_heads, self.dim_per_head = dim, num_heads, dim // num_heads
        self.is_first, self.is_last = is_first, is_last
        self.attn = EdgeMultiheadAttention(dim, num_heads, _act(attn_act))
        if is_first:
            self.output_proj, self.vec_proj = nn.Linear(dim, dim), None
        elif is_last:
            self.output_proj, self.vec_proj = nn.Linear(dim, 2 * dim), nn.Linear(dim, 2 * dim, bias=False)
        else:
            self.output_proj, self.vec_proj = nn.Linear(dim, 3 * dim), nn.Linear(dim, 3 * dim, bias=False)

    def forward(self, x, edge_feat, edge_vec, node_vec, center, neighbor, envelope, n):
        values, gate = self.attn(x, center, neighbor, envelope)
        scal = scatter_sum(values * edge_feat * gate.unsqueeze(-1), center, n).flatten(-2)
        vmsg = None if self.is_last else scatter_sum(values.unsqueeze(-3) * edge_vec, center, n).flatten(-2)
        if self.is_first:
            return self.output_proj(scal), vmsg
        mixed, proj = self.vec_proj(node_vec), self.output_proj(scal)
        if self.is_last:
            left, right = torch.split(mixed, self.dim, -1)
            scale, shift = torch.split(proj, self.dim, -1)
            return (left * right).sum(-2) * scale + shift, None
        left, right, carry = torch.split(mixed, self.dim, -1)
        vgate, scale, shift = torch.split(proj, self.dim, -1)
        return (left * right).sum(-2) * scale + shift, carry * vgate.unsqueeze(-2) + vmsg


class D3CSODispersion(nn.Module):
    """D3 two-body dispersion with the C6-only CSO damping ``s6 + a1 / (1 + exp(r - 2.5 R0))`` over
    ``1 / (r^6 + r_c^6)`` (kcal/mol, graph edges within ``disp_cutoff``)."""

    def __init__(self, s6: float = 1.0, a1: float = 0.86, rc_bohr: float = 7.75, disp_cutoff: Optional[float] = 10.0,
                 references: str = "2010"):
        super().__init__()
        self.s6, self.a1, self.rc_bohr, self.disp_cutoff = s6, a1, rc_bohr, disp_cutoff
        c6ab, rcov, r2r4 = d3_legacy.legacy_tables(str(references))
        dt = torch.get_default_dtype()
        self.register_buffer("_c6ab", c6ab.to(dt), persistent=False)
        self.register_buffer("_rcov", rcov.to(dt), persistent=False)
        self.register_buffer("_r2r4", r2r4.to(dt), persistent=False)

    def forward(self, z: Tensor, edge_vec: Tensor, edge_index: Tensor, n: int) -> Tensor:
        j, i = edge_index[0], edge_index[1]
        r = torch.linalg.norm(edge_vec, dim=-1) / d3_legacy.AUTOANG
        cut = None if self.disp_cutoff is None else self.disp_cutoff / d3_legacy.AUTOANG
        zi, zj = z[i], z[j]
        cn = d3_legacy.coordination(zi, zj, r, i, n, cut, self._rcov)
        c6 = d3_legacy.pair_c6(zi, zj, cn[i], cn[j], self._c6ab)
        r0 = torch.sqrt(3.0 * self._r2r4[zi].to(c6.dtype) * self._r2r4[zj].to(c6.dtype))
        e = -0.5 * c6 * (self.s6 + self.a1 / (1.0 + torch.exp(r - 2.5 * r0))) / (r ** 6 + self.rc_bohr ** 6)
        if cut is not None:
            e = torch.where(r < cut, e, torch.zeros_like(e))
        return r.new_zeros(n).index_add(0, i, e) * HARTREE_KCAL_MOL


@register_model("bamboo")
class BAMBOO(InteratomicPotential):
    head_modules = ("energy_mlp",)

    def __init__(self, dim: int = 64, num_rbf: int = 32, cutoff: float = 5.0, n_layers: int = 3, num_heads: int = 16,
                 charge_ub: float = 2.0, charge_mlp_layers: int = 2, energy_mlp_layers: int = 2, n_elements: int = 87,
                 act_fn="silu", attn_act_fn="gelu", coul_damping_beta: float = 18.7, coul_damping_r0: float = 2.2,
                 ele_factor: float = ELE_FACTOR, use_electrostatics: bool = True, use_dispersion: bool = False,
                 disp_cutoff: float = 10.0, d3_references: str = "2010", species=None):
        super().__init__()
        if n_layers < 2:
            raise ValueError("n_layers (n_interactions) must be >= 2")
        if dim % num_heads:
            raise ValueError(f"dim ({dim}) must be divisible by num_heads ({num_heads})")
        self.cutoff, self.dim, self.num_rbf, self.n_layers, self.num_heads = cutoff, dim, num_rbf, n_layers, num_heads
        self.charge_ub, self.n_elements, self.ele_factor = charge_ub, n_elements, ele_factor
        self.coul_damping_beta, self.coul_damping_r0 = coul_damping_beta, coul_damping_r0
        self.use_electrostatics, self.use_dispersion = use_electrostatics, use_dispersion
        self.species = list(species) if species is not None else None
        self.node_feature_dim = dim
        self.atom_emb = nn.Embedding(n_elements, dim)
        self.dis_rbf = ExpNormalSmearing(num_rbf, cutoff, trainable=True)
        self.cutoff_fn = CosineCutoff(cutoff)
        self.rbf_proj = nn.Sequential(nn.Linear(num_rbf, dim, bias=False), _act(attn_act_fn))
        layers = [GETLayer(dim, num_heads, attn_act_fn, is_first=True)]
        layers += [GETLayer(dim, num_heads, attn_act_fn) for _ in range(n_layers - 2)]
        layers.append(GETLayer(dim, num_heads, attn_act_fn, is_last=True))
        self.layers = nn.ModuleList(layers)
        self.energy_mlp = _energy_mlp(energy_mlp_layers, dim, act_fn)
        self.charge_mlp = _energy_mlp(charge_mlp_layers, dim, act_fn)
        self.electronegativity_mlp = _energy_mlp(charge_mlp_layers, dim, act_fn)
        self.hardness_mlp = _energy_mlp(charge_mlp_layers, dim, act_fn)
        self.coul_softplus = nn.Softplus(beta=coul_damping_beta)
        self.dispersion = D3CSODispersion(disp_cutoff=disp_cutoff, references=str(d3_references)) \
            if use_dispersion else None

    def receptive_field(self):
        return None if self.use_electrostatics else self.n_layers * self.cutoff

    def coulomb_energy(self, q: Tensor, vec: Tensor, row: Tensor, col: Tensor) -> Tensor:
        d = torch.linalg.norm(vec, dim=-1)
        r0 = self.coul_damping_r0
        return self.ele_factor * q[row] * q[col] / d * d / r0 / (1.0 + self.coul_softplus((d - r0) / r0))

    def _evaluate(self, z, edge_index, edge_vec, pos, batch, num_graphs, total_charge):
        n = z.shape[0]
        center, neighbor = edge_index[1], edge_index[0]
        r = torch.linalg.norm(edge_vec, dim=-1)
        unit = edge_vec / r.unsqueeze(-1)
        envelope = self.cutoff_fn(r)
        edge_feat = self.rbf_proj(self.dis_rbf(r)).unflatten(-1, (self.num_heads, self.dim // self.num_heads))
        edge_vec_feat = unit[..., None, None] * edge_feat.unsqueeze(-3)
        x0 = self.atom_emb(z)
        chi, hard = self.electronegativity_mlp(x0).squeeze(-1), self.hardness_mlp(x0).squeeze(-1)
        x, v = x0, None
        for layer in self.layers:
            dx, dv = layer(x, edge_feat, edge_vec_feat, v, center, neighbor, envelope, n)
            x = x + dx
            if dv is not None:
                v = dv if v is None else v + dv
        q = self.charge_ub * torch.tanh(self.charge_mlp(x).squeeze(-1) / self.charge_ub)
        n_per = scatter_sum(torch.ones_like(q), batch, num_graphs)
        q = q + ((total_charge.to(q.dtype) - scatter_sum(q, batch, num_graphs)) / n_per)[batch]
        node_nn = self.energy_mlp(x).squeeze(-1)
        node = node_nn
        node_elec = torch.zeros_like(node_nn)
        if self.use_electrostatics:
            node_elec = chi ** 2 * q + hard ** 2 * q ** 2
            row, col = all_pairs(batch)
            if row.numel():
                pv = (pos[row] - pos[col]).to(q.dtype)
                node_elec = node_elec + 0.5 * scatter_sum(self.coulomb_energy(q, pv, row, col), row, n)
            node = node + node_elec
        if self.dispersion is not None:
            node = node + self.dispersion(z, edge_vec, edge_index, n)
        return x, node, q, node_nn, node_elec

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        if self.use_electrostatics:
            raise RuntimeError("BAMBOO with electrostatics needs whole structures (positions and net charge)")
        n = atomic_numbers.shape[0]
        out = self._evaluate(atomic_numbers, edge_index, edge_vec, edge_vec.new_zeros(n, 3),
                             torch.zeros(n, dtype=torch.long, device=edge_vec.device), 1, edge_vec.new_zeros(1))
        return out[0], out[1]

    def forward(self, data: AtomicGraph) -> dict:
        b = data.num_graphs
        vec = data.edge_vectors()
        total = data.total_charge if data.total_charge is not None else vec.new_zeros(b)
        x, node, q, node_nn, node_elec = self._evaluate(data.atomic_numbers, data.edge_index, vec, data.pos,
                                                        data.batch, b, total)
        e_nn = self.aggregate_energy(node_nn, data)
        e_elec = self.aggregate_energy(node_nn + node_elec, data) - e_nn if self.use_electrostatics else \
            torch.zeros(b, dtype=torch.float64, device=vec.device)
        return {"node_energy": node, "energy": self.aggregate_energy(node, data), "node_features": x, "charges": q,
                "dipole": scatter_sum(q.unsqueeze(-1) * data.pos.to(q.dtype), data.batch, b) / DEBYE_EA,
                "energy_nn": e_nn, "energy_elec": e_elec}

    @classmethod
    def from_config(cls, cfg) -> "BAMBOO":
        e = dict(cfg.extra or {})
        keys = ("num_heads", "charge_ub", "charge_mlp_layers", "energy_mlp_layers", "n_elements", "act_fn",
                "attn_act_fn", "coul_damping_beta", "coul_damping_r0", "ele_factor", "use_electrostatics",
                "use_dispersion", "disp_cutoff", "d3_references", "species")
        return cls(dim=cfg.n_features, num_rbf=cfg.n_rbf, cutoff=cfg.cutoff, n_layers=cfg.n_interactions,
                   **{k: e[k] for k in keys if k in e})
