"""GemNet (Gasteiger, Becker & Guennemann, NeurIPS 2021): geometric message passing with
triplets (GemNet-T) and quadruplets (GemNet-Q), optional direct (non-conservative) forces
(GemNet-dT / dQ).

Edge messages ``m_ca`` exchange information over triplets ``b -> a <- c`` (angle at ``a``,
spherical Fourier-Bessel basis) and over quadruplets ``d -> b -> a <- c`` within an interaction
cutoff (dihedral-resolved real spherical harmonics); every interaction is a Hadamard radial gate,
a down projection, the neighbour sums against the angular basis, a radial-mixed bilinear map and
up projections of both directions; residual stacks scaled by ``1/sqrt(2)``; atom updates and
per-block outputs; fitted scale factors (variance matching). Index plans, options and parameter
names follow the reference (``src/xnn/gnn/models/gemnet.py``) so that weights and fitted scale
factors transplant.

The neighbour sums scatter the outer products of the angular basis and the gathered features onto
the output edges (no padded ``(E, k_max, ...)`` tables).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..featurizers.spherical_bessel import SphericalBesselBasis, real_spherical_harmonics, zonal_harmonics
from ..nn.cutoff import PolynomialCutoff
from ..nn.radial import BesselRBF
from ..ops.scatter import scatter_sum
from .base import InteratomicPotential
from .registry import register_model

_MAX_Z = 100
_IS2, _IS3 = 1.0 / math.sqrt(2.0), 1.0 / math.sqrt(3.0)


def he_orthogonal_(w: Tensor) -> Tensor:
    """An orthogonal matrix standardised per output unit to variance ``1 / fan_in``."""
    with torch.no_grad():
        nn.init.orthogonal_(w)
        var, mean = torch.var_mean(w, dim=1, unbiased=True, keepdim=True)
        w.sub_(mean).div_(torch.sqrt(var + 1e-6)).mul_(w.shape[1] ** -0.5)
    return w


class _Dense(nn.Linear):
    """Bias-free linear layer, ``silu(x) / 0.6`` when activated."""

    def __init__(self, n_in: int, n_out: int, activation: bool = False, init: str = "he_orthogonal"):
        super().__init__(n_in, n_out, bias=False)
        self.activation = activation
        if init == "zeros":
            nn.init.zeros_(self.weight)
        elif init == "he_orthogonal":
            he_orthogonal_(self.weight)
        else:
            raise ValueError(f"init must be 'he_orthogonal' or 'zeros', got {init!r}")

    def forward(self, x: Tensor) -> Tensor:
        y = nn.functional.linear(x, self.weight)
        return nn.functional.silu(y) * (1.0 / 0.6) if self.activation else y


class _Residual(nn.Module):
    def __init__(self, n: int):
        super().__init__()
        self.lin1, self.lin2 = _Dense(n, n, True), _Dense(n, n, True)

    def forward(self, x: Tensor) -> Tensor:
        return (x + self.lin2(self.lin1(x))) * _IS2


class ScaleFactor(nn.Module):
    """``y * scale``; while fitting it accumulates the variances of a reference and of ``y``."""

    def __init__(self):
        super().__init__()
        self.register_buffer("scale_factor", torch.tensor(1.0))
        self.register_buffer("stats", torch.zeros(3, dtype=torch.float64), persistent=False)
        self.fitting = False

    def forward(self, ref: Tensor, y: Tensor) -> Tensor:
        y = y * self.scale_factor
        if self.fitting and ref.shape[0] > 1 and y.shape[0] > 1:
            n = float(y.shape[0])
            vr = torch.var(ref.detach(), dim=0).mean().double()
            vy = torch.var(y.detach(), dim=0).mean().double()
            self.stats.add_(torch.stack([vr * n, vy * n, torch.ones_like(vy) * n]))
        return y


class _EdgeEmbedding(nn.Module):
    def __init__(self, n_atom: int, n_in: int, n_out: int):
        super().__init__()
        self.dense = _Dense(2 * n_atom + n_in, n_out, True)

    def forward(self, h: Tensor, x: Tensor, src: Tensor, dst: Tensor) -> Tensor:
        return self.dense(torch.cat([h[src], h[dst], x], -1))


class _AtomUpdate(nn.Module):
    def __init__(self, n_atom: int, n_edge: int, n_rbf_emb: int, n_residual: int):
        super().__init__()
        self.lin_rbf = _Dense(n_rbf_emb, n_edge)
        self.scale_sum = ScaleFactor()
        self.dense = _Dense(n_edge, n_atom, True)
        self.residuals = _stack(n_residual, n_atom)

    def forward(self, m: Tensor, rbf: Tensor, dst: Tensor, n: int):
        gated = m * self.lin_rbf(rbf)
        h = self.dense(self.scale_sum(m, scatter_sum(gated, dst, n)))
        for res in self.residuals:
            h = res(h)
        return h, gated


class _ForceHead(nn.Module):
    def __init__(self, n_edge: int, n_residual: int, output_init: str):
        super().__init__()
        self.scale_rbf = ScaleFactor()
        self.dense = _Dense(n_edge, n_edge, True)
        self.residuals = _stack(n_residual, n_edge)
        self.final = _Dense(n_edge, 1, init=output_init)

    def forward(self, m: Tensor, gated: Tensor) -> Tensor:
        x = self.dense(self.scale_rbf(m, gated))
        for res in self.residuals:
            x = res(x)
        return self.final(x).squeeze(-1)


class _Output(nn.Module):
    def __init__(self, n_atom, n_edge, n_rbf_emb, n_residual, output_init, direct_forces):
        super().__init__()
        self.atom = _AtomUpdate(n_atom, n_edge, n_rbf_emb, n_residual)
        self.final = _Dense(n_atom, 1, init=output_init)
        self.forces = _ForceHead(n_edge, n_residual, output_init) if direct_forces else None

    def forward(self, m, rbf, dst, n):
        h, gated = self.atom(m, rbf, dst, n)
        f = self.forces(m, gated) if self.forces is not None else m.new_zeros(0)
        return h, self.final(h).squeeze(-1), f


def _basis_sums(x: Tensor, sph: Tensor, out: Tensor, n_out: int) -> Tensor:
    """``sum_{t: out_t = e} sph_t (x) x_t`` per output edge, ``(n_out, L, F)``."""
    return scatter_sum(sph[:, :, None] * x[:, None, :], out, n_out)


def _mix(summed: Tensor, rad: Tensor, weight: Tensor) -> Tensor:
    mixed = torch.bmm(rad, summed)                       # (E, J, F)
    j, f = weight.shape[0], summed.shape[2]
    return mixed.reshape(summed.shape[0], j * f) @ weight.reshape(j * f, weight.shape[2])


def _bilinear_init_(w: Tensor) -> None:
    j, fi, fo = w.shape
    flat = he_orthogonal_(torch.empty(fo, j * fi, dtype=w.dtype))
    with torch.no_grad():
        w.copy_(flat.t().reshape(j, fi, fo))


def _stack(n: int, width: int) -> nn.ModuleList:
    return nn.ModuleList(_Residual(width) for _ in range(n))


class _ManyBody(nn.Module):
    """The skeleton shared by the triplet and quadruplet interactions: an edge update gated by the
    radial basis, a projection down to the interaction width, a bilinear contraction of the
    basis sums, and up-projections for the edge and for its reverse (averaged)."""

    first: str

    def _build(self, n_edge: int, n_down: int, n_rbf_emb: int, n_bilinear_basis: int, n_bilinear: int,
               scale_names) -> None:
        setattr(self, self.first, _Dense(n_edge, n_edge, True))
        self.lin_rbf = _Dense(n_rbf_emb, n_edge)
        self.down = _Dense(n_edge, n_down, True)
        self.bilinear = nn.Parameter(torch.empty(n_bilinear_basis, n_down, n_bilinear))
        _bilinear_init_(self.bilinear)
        for name in scale_names:
            setattr(self, name, ScaleFactor())
        self.up_ca, self.up_ac = (_Dense(n_bilinear, n_edge, True) for _ in range(2))

    def _gated_down(self, m: Tensor, rbf: Tensor) -> Tensor:
        x = getattr(self, self.first)(m)
        return self.down(self.scale_rbf(x, x * self.lin_rbf(rbf)))

    def _up(self, y: Tensor, rev: Tensor) -> Tensor:
        return (self.up_ca(y) + self.up_ac(y).index_select(0, rev)) * _IS2


class _TripletInteraction(_ManyBody):
    first = "dense_ba"

    def __init__(self, n_edge, n_trip, n_rbf_emb, n_cbf_emb, n_bilinear):
        super().__init__()
        self._build(n_edge, n_trip, n_rbf_emb, n_cbf_emb, n_bilinear, ("scale_rbf", "scale_cbf_sum"))

    def forward(self, m, rbf, cbf_rad, sph, t_out, t_in, rev):
        x = self._gated_down(m, rbf).index_select(0, t_in)
        y = self.scale_cbf_sum(x, _mix(_basis_sums(x, sph, t_out, m.shape[0]), cbf_rad, self.bilinear))
        return self._up(y, rev)


class _QuadrupletInteraction(_ManyBody):
    first = "dense_db"

    def __init__(self, n_edge, n_quad, n_rbf_emb, n_cbf_emb, n_sbf_emb, n_bilinear):
        super().__init__()
        self._build(n_edge, n_quad, n_rbf_emb, n_sbf_emb, n_bilinear, ("scale_rbf", "scale_cbf", "scale_sbf_sum"))
        self.lin_cbf = _Dense(n_cbf_emb, n_quad)

    def forward(self, m, rbf, cbf, sbf_rad, sph, intm_db, q_out, q_intm, rev):
        x = self._gated_down(m, rbf).index_select(0, intm_db)
        x = self.scale_cbf(x, x * self.lin_cbf(cbf)).index_select(0, q_intm)
        y = self.scale_sbf_sum(x, _mix(_basis_sums(x, sph, q_out, m.shape[0]), sbf_rad, self.bilinear))
        return self._up(y, rev)


class _Interaction(nn.Module):
    def __init__(self, n_atom, n_edge, n_trip, n_quad, n_rbf_emb, n_cbf_emb, n_sbf_emb, n_bil_trip, n_bil_quad,
                 n_before, n_after, n_concat, n_atom_residual, quadruplets):
        super().__init__()
        self.dense_ca = _Dense(n_edge, n_edge, True)
        self.quad = (_QuadrupletInteraction(n_edge, n_quad, n_rbf_emb, n_cbf_emb, n_sbf_emb, n_bil_quad)
                     if quadruplets else None)
        self.trip = _TripletInteraction(n_edge, n_trip, n_rbf_emb, n_cbf_emb, n_bil_trip)
        self.before_skip, self.after_skip = _stack(n_before, n_edge), _stack(n_after, n_edge)
        self.atom_update = _AtomUpdate(n_atom, n_edge, n_rbf_emb, n_atom_residual)
        self.concat = _EdgeEmbedding(n_atom, n_edge, n_edge)
        self.residual_m = _stack(n_concat, n_edge)

    def forward(self, h, m, src, dst, rev, g3, g4, rbf_h):
        x_skip = self.dense_ca(m)
        x3 = self.trip(m, *g3, rev)
        if self.quad is not None:
            x = (x_skip + x3 + self.quad(m, *g4, rev)) * _IS3
        else:
            x = (x_skip + x3) * _IS2
        for res in self.before_skip:
            x = res(x)
        m = (m + x) * _IS2
        for res in self.after_skip:
            m = res(m)
        h_new, _ = self.atom_update(m, rbf_h, dst, h.shape[0])
        h = (h + h_new) * _IS2
        m_new = self.concat(h, m, src, dst)
        for res in self.residual_m:
            m_new = res(m_new)
        return h, (m + m_new) * _IS2


def _lexsort(cols: List[Tensor]) -> Tensor:
    idx = torch.arange(cols[0].shape[0], device=cols[0].device)
    for c in reversed(cols):
        idx = idx[torch.sort(c[idx], stable=True)[1]]
    return idx


def reverse_edges(edge_index: Tensor, edge_vec: Tensor) -> Tensor:
    """The index of every edge's reverse (same atoms swapped, exactly negated vector)."""
    src, dst = edge_index[0], edge_index[1]
    fwd = _lexsort([src, dst, edge_vec[:, 0], edge_vec[:, 1], edge_vec[:, 2]])
    bwd = _lexsort([dst, src, -edge_vec[:, 0], -edge_vec[:, 1], -edge_vec[:, 2]])
    rev = torch.empty_like(fwd)
    rev[bwd] = fwd
    ok = (src[rev] == dst) & (dst[rev] == src) & (edge_vec[rev] == -edge_vec).all(-1)
    if not bool(ok.all()):
        raise RuntimeError("GemNet needs a neighbor list that contains the reverse of every edge with the exactly "
                           "negated edge vector")
    return rev


def triplets(edge_index: Tensor, num_nodes: int) -> Tuple[Tensor, Tensor]:
    """``(ca, ba)``: every pair of distinct edges into the same atom ``a``."""
    dst = edge_index[1]
    order = torch.sort(dst, stable=True)[1]
    counts = torch.bincount(dst, minlength=num_nodes)
    starts = torch.cumsum(counts, 0) - counts
    n_in = counts[dst]
    ca = torch.repeat_interleave(torch.arange(dst.shape[0], device=dst.device), n_in)
    local = torch.arange(ca.shape[0], device=dst.device) - torch.repeat_interleave(torch.cumsum(n_in, 0) - n_in, n_in)
    ba = order[starts[dst[ca]] + local]
    keep = ba != ca
    return ca[keep], ba[keep]


def quadruplet_indices(src, dst, vec, emb_ids, edge_index, edge_vec, r_all, rev_all, num_nodes, int_cutoff) -> dict:
    """Quadruplets ``d -> b -> a <- c``: the interaction edge ``b -> a`` (within ``int_cutoff``), an
    embedding edge ``d -> b`` (not its reverse) and an embedding edge ``c -> a`` (not the interaction
    edge itself), ``c`` and ``d`` distinct images; grouped by the output edge ``c -> a``."""
    int_ids = torch.nonzero(r_all <= int_cutoff).flatten()
    b, a = edge_index[0][int_ids], edge_index[1][int_ids]
    v_ba = edge_vec[int_ids]
    order = torch.sort(dst, stable=True)[1]
    counts = torch.bincount(dst, minlength=num_nodes)
    starts = torch.cumsum(counts, 0) - counts
    n_a, n_b = counts[a], counts[b]
    ar = torch.arange(int_ids.shape[0], device=src.device)
    intm_q = torch.repeat_interleave(ar, n_b)
    intm_first = torch.cumsum(n_b, 0) - n_b
    intm_db = order[starts[b][intm_q] + torch.arange(intm_q.shape[0], device=src.device) - intm_first[intm_q]]
    n_q = n_a * n_b
    quad_q = torch.repeat_interleave(ar, n_q)
    local = torch.arange(quad_q.shape[0], device=src.device) - (torch.cumsum(n_q, 0) - n_q)[quad_q]
    nb_q = n_b[quad_q]
    ia, ib = torch.div(local, nb_q, rounding_mode="floor"), torch.remainder(local, nb_q)
    ca = order[starts[a][quad_q] + ia]
    q_intm = intm_first[quad_q] + ib
    db = intm_db[q_intm]
    cd = v_ba[quad_q] + vec[db] - vec[ca]
    same = (src[ca] == src[db]) & ((cd * cd).sum(-1) < 1e-8)
    keep = (emb_ids[ca] != int_ids[quad_q]) & (emb_ids[db] != rev_all[int_ids][quad_q]) & ~same
    ca, quad_q, q_intm = ca[keep], quad_q[keep], q_intm[keep]
    perm = torch.sort(ca, stable=True)[1]
    return {"int_ids": int_ids, "intm_q": intm_q, "intm_db": intm_db, "quad_q": quad_q[perm], "q_out": ca[perm],
            "q_intm": q_intm[perm]}


def index_plan(edge_index, edge_vec, num_nodes, emb_cutoff, int_cutoff, quadruplets) -> Dict[str, Tensor]:
    r_all = torch.linalg.norm(edge_vec, dim=-1)
    rev_all = reverse_edges(edge_index, edge_vec)
    emb_ids = torch.nonzero(r_all <= emb_cutoff).flatten()
    in_emb = torch.full_like(r_all, -1, dtype=torch.long)
    in_emb[emb_ids] = torch.arange(emb_ids.shape[0], device=emb_ids.device)
    src, dst = edge_index[0][emb_ids], edge_index[1][emb_ids]
    t_out, t_in = triplets(torch.stack([src, dst]), num_nodes)
    plan = {"emb_ids": emb_ids, "rev": in_emb[rev_all[emb_ids]], "t_out": t_out, "t_in": t_in}
    if quadruplets:
        plan.update(quadruplet_indices(src, dst, edge_vec[emb_ids], emb_ids, edge_index, edge_vec, r_all, rev_all,
                                       num_nodes, int_cutoff))
    return plan


@register_model("gemnet")
class GemNet(InteratomicPotential):
    head_modules = ("outputs", "atom_ref")

    def __init__(self, n_features: int = 128, n_edge_features: int = 128, n_interactions: int = 4, n_rbf: int = 6,
                 n_spherical: int = 7, cutoff: float = 5.0, int_cutoff: float = 10.0, p: int = 5,
                 n_triplet_features: int = 64, n_quadruplet_features: int = 32, n_rbf_features: int = 16,
                 n_cbf_features: int = 16, n_sbf_features: int = 32, n_bilinear_triplet: int = 64,
                 n_bilinear_quadruplet: int = 32, n_before_skip: int = 1, n_after_skip: int = 1, n_concat: int = 1,
                 n_atom_residual: int = 2, quadruplets: bool = True, direct_forces: bool = False,
                 forces_coupled: bool = False, output_init: str = "he_orthogonal", trainable_rbf: bool = True,
                 species=None, atomic_energies=None):
        super().__init__()
        if output_init not in ("he_orthogonal", "zeros"):
            raise ValueError(f"output_init must be 'he_orthogonal' or 'zeros', got {output_init!r}")
        self.quadruplets, self.direct_forces, self.forces_coupled = bool(quadruplets), bool(direct_forces), bool(
            forces_coupled)
        self.emb_cutoff, self.int_cutoff = float(cutoff), float(int_cutoff)
        self.cutoff = max(self.emb_cutoff, self.int_cutoff) if self.quadruplets else self.emb_cutoff
        self.n_spherical, self.n_rbf, self.node_feature_dim = n_spherical, n_rbf, n_features
        if species is not None:
            self.species = [int(z) for z in species]
        self.rbf = BesselRBF(n_rbf, cutoff, trainable=trainable_rbf)
        self.envelope = PolynomialCutoff(cutoff, p)
        self.cbf = SphericalBesselBasis(n_spherical, n_rbf, cutoff)
        self.int_envelope = PolynomialCutoff(int_cutoff, p)
        self.cbf_int = SphericalBesselBasis(n_spherical, n_rbf, int_cutoff)
        n_cbf = n_spherical * n_rbf
        self.lin_rbf3 = _Dense(n_rbf, n_rbf_features)
        self.lin_cbf3 = _Dense(n_cbf, n_cbf_features)
        self.lin_rbf_h = _Dense(n_rbf, n_rbf_features)
        self.lin_rbf_out = _Dense(n_rbf, n_rbf_features)
        self.lin_rbf4 = self.lin_cbf4 = self.lin_sbf4 = None
        if self.quadruplets:
            self.lin_rbf4 = _Dense(n_rbf, n_rbf_features)
            self.lin_cbf4 = _Dense(n_cbf, n_cbf_features)
            self.lin_sbf4 = _Dense(n_spherical ** 2 * n_rbf, n_sbf_features)
        self.register_buffer("sbf_degree", torch.repeat_interleave(torch.arange(n_spherical),
                                                                   2 * torch.arange(n_spherical) + 1), persistent=False)
        self.atom_embedding = nn.Embedding(_MAX_Z, n_features)
        nn.init.uniform_(self.atom_embedding.weight, -math.sqrt(3.0), math.sqrt(3.0))
        self.edge_embedding = _EdgeEmbedding(n_features, n_rbf, n_edge_features)
        self.interactions = nn.ModuleList([
            _Interaction(n_features, n_edge_features, n_triplet_features, n_quadruplet_features, n_rbf_features,
                         n_cbf_features, n_sbf_features, n_bilinear_triplet, n_bilinear_quadruplet, n_before_skip,
                         n_after_skip, n_concat, n_atom_residual, self.quadruplets) for _ in range(n_interactions)])
        self.outputs = nn.ModuleList([_Output(n_features, n_edge_features, n_rbf_features, n_atom_residual, output_init,
                                              self.direct_forces) for _ in range(n_interactions + 1)])
        self.atom_ref = nn.Embedding(_MAX_Z, 1)
        nn.init.zeros_(self.atom_ref.weight)
        self.register_buffer("scaling_fitted", torch.tensor(False))
        if atomic_energies is not None:
            if species is None:
                raise ValueError("species is required to map atomic_energies")
            self.set_atomic_energies(species, atomic_energies)

    def set_atomic_energies(self, species, values) -> None:
        with torch.no_grad():
            self.atom_ref.weight[torch.tensor(list(species)), 0] = torch.as_tensor(values,
                                                                                   dtype=self.atom_ref.weight.dtype)

    def receptive_field(self) -> float:
        return (len(self.interactions) + 1) * self.cutoff

    @property
    def forms_forces_directly(self) -> bool:
        return self.direct_forces

    def _quadruplet_angles(self, vec, r, v_ba, r_ba, plan):
        intm_q, intm_db, quad_q, ca = plan["intm_q"], plan["intm_db"], plan["quad_q"], plan["q_out"]
        db = intm_db[plan["q_intm"]]
        cos_abd = -(v_ba[intm_q] * vec[intm_db]).sum(-1) / (r_ba[intm_q] * r[intm_db])
        axis = -v_ba[quad_q] / r_ba[quad_q][:, None]
        u_c = -vec[ca] / r[ca][:, None]
        to_d = -vec[db]
        p_d = to_d - (to_d * axis).sum(-1, keepdim=True) * axis
        norm_d = torch.sqrt(torch.clamp((p_d * p_d).sum(-1), min=1e-18))
        e_x = p_d / norm_d[:, None]
        e_y = torch.cross(axis, e_x, dim=-1)
        z = (u_c * axis).sum(-1).clamp(-1.0, 1.0)
        x, y = (u_c * e_x).sum(-1), (u_c * e_y).sum(-1).abs()
        flat = norm_d <= 1e-9
        x = torch.where(flat, torch.zeros_like(x), x)
        y = torch.where(flat, torch.sqrt(torch.clamp(1.0 - z * z, min=1e-18)), y)
        return cos_abd, real_spherical_harmonics(self.n_spherical - 1, x, y, z)

    def _evaluate(self, z: Tensor, edge_index: Tensor, edge_vec: Tensor):
        n = z.shape[0]
        plan = index_plan(edge_index, edge_vec.detach(), n, self.emb_cutoff, self.int_cutoff, self.quadruplets)
        r_all = torch.linalg.norm(edge_vec, dim=-1)
        emb_ids, rev = plan["emb_ids"], plan["rev"]
        src, dst = edge_index[0][emb_ids], edge_index[1][emb_ids]
        vec, r = edge_vec[emb_ids], r_all[emb_ids]
        t_out, t_in = plan["t_out"], plan["t_in"]
        L, N = self.n_spherical, self.n_rbf
        env = self.envelope(r)
        rbf = self.rbf(r) * env[:, None]
        rad = self.cbf.radial(r) * env[:, None, None]
        cos_cab = ((vec[t_out] * vec[t_in]).sum(-1) / (r[t_out] * r[t_in])).clamp(-1.0, 1.0)
        cbf3_rad = torch.einsum("eln,jln->ejl", rad, self.lin_cbf3.weight.reshape(-1, L, N))
        g3 = (self.lin_rbf3(rbf), cbf3_rad, zonal_harmonics(L - 1, cos_cab), t_out, t_in)
        g4 = None
        if self.quadruplets:
            int_ids = plan["int_ids"]
            v_ba, r_ba = edge_vec[int_ids], r_all[int_ids]
            cos_abd, sph4 = self._quadruplet_angles(vec, r, v_ba, r_ba, plan)
            rad_ba = self.cbf_int.radial(r_ba) * self.int_envelope(r_ba)[:, None, None]
            y_abd = zonal_harmonics(L - 1, cos_abd.clamp(-1.0, 1.0))
            cbf4 = self.lin_cbf4((rad_ba[plan["intm_q"]] * y_abd[:, :, None]).reshape(-1, L * N))
            sbf_rad = torch.einsum("ekn,jkn->ejk", rad[:, self.sbf_degree], self.lin_sbf4.weight.reshape(-1, L * L, N))
            g4 = (self.lin_rbf4(rbf), cbf4, sbf_rad, sph4, plan["intm_db"], plan["q_out"], plan["q_intm"])
        rbf_h, rbf_out = self.lin_rbf_h(rbf), self.lin_rbf_out(rbf)
        h = self.atom_embedding(z)
        m = self.edge_embedding(h, rbf, src, dst)
        messages = [m]
        for blk in self.interactions:
            h, m = blk(h, m, src, dst, rev, g3, g4, rbf_h)
            messages.append(m)
        feats = h.new_zeros(n, self.node_feature_dim)
        node = self.atom_ref(z).squeeze(-1)
        edge_force = vec.new_zeros(vec.shape[0])
        for i, out in enumerate(self.outputs):
            ho, t, f = out(messages[i], rbf_out, dst, n)
            feats, node = feats + ho, node + t
            if self.direct_forces:
                edge_force = edge_force + f
        forces = vec.new_zeros(0, 3)
        if self.direct_forces:
            if self.forces_coupled:
                edge_force = 0.5 * (edge_force + edge_force[rev])
            forces = scatter_sum(edge_force[:, None] * vec / r[:, None], dst, n)
        return feats, node, forces

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        if self.direct_forces:
            raise RuntimeError("a GemNet with direct_forces has no energy-only core")
        f, e, _ = self._evaluate(atomic_numbers, edge_index, edge_vec)
        return f, e

    def node_energy(self, atomic_numbers, edge_index, edge_vec):
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> dict:
        f, e, forces = self._evaluate(data.atomic_numbers, data.edge_index, data.edge_vectors())
        out = {"node_energy": e, "energy": self.aggregate_energy(e, data), "node_features": f}
        if self.direct_forces:
            out["forces"] = forces.to(data.pos.dtype)
        return out

    def scale_factors(self) -> Dict[str, ScaleFactor]:
        names: Dict[str, ScaleFactor] = {}

        def output(i):
            names[f"OutBlock_{i}_sum"] = self.outputs[i].atom.scale_sum
            if self.outputs[i].forces is not None:
                names[f"OutBlock_{i}_had"] = self.outputs[i].forces.scale_rbf
        output(0)
        for i, blk in enumerate(self.interactions, start=1):
            if blk.quad is not None:
                names[f"QuadInteraction_{i}_had_rbf"] = blk.quad.scale_rbf
                names[f"QuadInteraction_{i}_had_cbf"] = blk.quad.scale_cbf
                names[f"QuadInteraction_{i}_sum_sbf"] = blk.quad.scale_sbf_sum
            names[f"TripInteraction_{i}_had_rbf"] = blk.trip.scale_rbf
            names[f"TripInteraction_{i}_sum_cbf"] = blk.trip.scale_cbf_sum
            names[f"AtomUpdate_{i}_sum"] = blk.atom_update.scale_sum
            output(i)
        return names

    def fit_scaling_factors(self, batches) -> Dict[str, float]:
        """Match, factor by factor in forward order, the output variance to its reference input."""
        batches = list(batches)
        fitted = {}
        was = self.training
        self.eval()
        for name, fac in self.scale_factors().items():
            fac.stats.zero_()
            fac.fitting = True
            try:
                with torch.no_grad():
                    for g in batches:
                        self(g)
            finally:
                fac.fitting = False
            vr, vy, cnt = fac.stats.tolist()
            if cnt == 0 or vy == 0:
                raise ValueError(f"no data reached the scaling factor {name}")
            with torch.no_grad():
                fac.scale_factor.mul_(math.sqrt(vr / vy))
            fitted[name] = float(fac.scale_factor)
        self.scaling_fitted.fill_(True)
        self.train(was)
        return fitted

    def load_scaling_factors(self, factors) -> None:
        if not isinstance(factors, dict):
            import json
            with open(factors) as f:
                factors = json.load(f)
        with torch.no_grad():
            for name, fac in self.scale_factors().items():
                if name not in factors:
                    raise KeyError(f"no value for the scaling factor {name}")
                fac.scale_factor.fill_(float(factors[name]))
        self.scaling_fitted.fill_(True)

    @classmethod
    def from_config(cls, cfg) -> "GemNet":
        e = dict(cfg.extra or {})
        quad = e.get("quadruplets")
        if quad is None:
            quad = not bool(e.get("triplets_only", False))
        init = str(e.get("output_init", "he_orthogonal")).lower()
        init = "he_orthogonal" if init == "heorthogonal" else init
        keys = ("n_edge_features", "n_spherical", "n_triplet_features", "n_quadruplet_features", "n_rbf_features",
                "n_cbf_features", "n_sbf_features", "n_bilinear_triplet", "n_bilinear_quadruplet", "n_before_skip",
                "n_after_skip", "n_concat", "n_atom_residual")
        model = cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, n_rbf=cfg.n_rbf, cutoff=cfg.cutoff,
                    int_cutoff=float(e.get("int_cutoff", 10.0)), p=int(e.get("p", e.get("envelope_exponent", 5))),
                    quadruplets=bool(quad), direct_forces=bool(e.get("direct_forces", False)),
                    forces_coupled=bool(e.get("forces_coupled", False)), output_init=init,
                    trainable_rbf=bool(e.get("trainable_rbf", True)), species=e.get("species"),
                    atomic_energies=e.get("atomic_energies"), **{k: int(e[k]) for k in keys if e.get(k) is not None})
        if e.get("scaling_factors") is not None:
            model.load_scaling_factors(e["scaling_factors"])
        return model
