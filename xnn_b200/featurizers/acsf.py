"""Behler atom-centred symmetry functions with a separate list per element (RuNNer conventions).

Every function has a central element, one neighbour element (radial) or an unordered pair of them
(angular), its parameters and one of the declared cutoff functions; an atom's descriptor is the
list of its element's functions (zero-padded to the longest list), optionally scaled by training
statistics. Types (``r_ij``, ``r_ik``, ``r_jk`` the distances of a neighbour pair ``j < k`` of
centre ``i``, ``theta`` the angle at ``i``, ``fc`` the function's cutoff):

* 1: ``sum_j fc(r_ij)^(2^(m-1))`` for ``m = 1 .. n_features``;
* 2: ``sum_j exp(-eta (r_ij - rs)^2) fc(r_ij)``;
* 3: ``2^(1-zeta) sum_{j<k} max(0, 1 + lambda cos theta)^zeta exp(-eta (r_ij^2 + r_ik^2 + r_jk^2))
  fc(r_ij) fc(r_ik) fc(r_jk)``;
* 8: ``sum_{j<k} g(theta) fc fc fc`` with ``g`` four Gaussians ``exp(-eta (theta - t)^2)`` at
  ``t = theta_s, 360 - theta_s, -theta_s, 360 + theta_s`` (degrees);
* 9: type 3 without the ``r_jk`` terms.

Cutoff kinds: ``cosine`` and ``tanh`` / ``tanh_approx`` with an inner radius, ``polynomial``
``(1 - r^2/r_c^2)^n`` and ``hard``. Scaling modes: ``none``, ``scale`` ``(G - min)/(max - min)``,
``center`` ``G - avg``, ``center_scale``, ``range`` (a function with ``max == min`` is not divided).
The specification format, buffer names and scaling statistics follow the reference
(``src/xnn/dnn/featurizers/acsf.py:1-711``) so that a RuNNer model read by either framework gives
the same descriptor. Evaluation: every edge (triplet) looks up the rows of its
(centre, neighbour[, neighbour]) species and evaluates them at once.
"""
from __future__ import annotations

import math
from typing import Iterable, List, Optional, Sequence, Tuple

import torch
from torch import Tensor, nn

from ..data.elements import ATOMIC_NUMBERS
from ..ops.scatter import build_center_pairs

CUTOFF_KINDS = ("cosine", "tanh", "tanh_approx", "polynomial", "hard")
SCALING_MODES = ("none", "scale", "center", "center_scale", "range")


def _as_z(value) -> int:
    return int(value) if not isinstance(value, str) else ATOMIC_NUMBERS[value]


def cutoff_function(r: Tensor, kind: str, r_cut: float, r_inner: float = 0.0, exponent: int = 2) -> Tensor:
    inside = r < r_cut
    if kind == "hard":
        return inside.to(r.dtype)
    if kind == "polynomial":
        val = (1.0 - (r / r_cut) ** 2) ** int(exponent)
        return torch.where(inside, val, torch.zeros_like(r))
    x = ((r - r_inner) / (r_cut - r_inner)).clamp(0.0, 1.0)
    if kind == "cosine":
        val = 0.5 * (torch.cos(math.pi * x) + 1.0)
    elif kind == "tanh":
        val = torch.tanh(1.0 - x) ** 3
    elif kind == "tanh_approx":
        y = 1.0 - x
        val = (y * (27.0 + y * y) / (27.0 + 9.0 * y * y)) ** 3
    else:
        raise ValueError(f"unknown cutoff kind {kind!r}; choose one of {CUTOFF_KINDS}")
    return torch.where(inside, val, torch.zeros_like(r))


def _acos_margin(dtype) -> float:
    return {torch.float64: 1e-15, torch.float32: 1.1920928955078125e-07, torch.bfloat16: 0.0078125}.get(
        dtype, 0.0009765625)


def _cutoff_spec(spec) -> dict:
    spec = dict(spec)
    kind = str(spec.get("kind", "cosine")).lower()
    if kind not in CUTOFF_KINDS:
        raise ValueError(f"unknown cutoff kind {kind!r}; choose one of {CUTOFF_KINDS}")
    out = {"kind": kind, "r_cut": float(spec["r_cut"]), "r_inner": float(spec.get("r_inner", 0.0) or 0.0),
           "exponent": int(spec.get("exponent", 2))}
    if out["r_inner"] >= out["r_cut"]:
        raise ValueError(f"cutoff {spec}: the inner radius must be below r_cut")
    if kind in ("polynomial", "hard") and out["r_inner"] != 0.0:
        raise ValueError(f"cutoff {spec}: the {kind} kind has no inner radius")
    return out


def _function_rows(spec, n_cutoffs: int) -> List[dict]:
    spec = dict(spec)
    t = int(spec["type"])
    if t not in (1, 2, 3, 8, 9):
        raise ValueError(f"unsupported symmetry function type {t} (1, 2, 3, 8 or 9)")
    nb = [_as_z(z) for z in spec["neighbors"]]
    if len(nb) != (1 if t in (1, 2) else 2):
        raise ValueError(f"type {t} takes {1 if t in (1, 2) else 2} neighbour element(s): {spec}")
    cut = int(spec.get("cutoff", 0))
    if not 0 <= cut < n_cutoffs:
        raise ValueError(f"function {spec} names cutoff {cut}; {n_cutoffs} are declared")
    row = {"element": _as_z(spec["element"]), "type": t, "neighbors": tuple(sorted(nb)), "cutoff": cut,
           "eta": float(spec.get("eta", 0.0)), "rs": float(spec.get("rs", 0.0)),
           "lambda": float(spec.get("lambda", 1.0)), "zeta": float(spec.get("zeta", 1.0)),
           "theta_s": float(spec.get("theta_s", 0.0)), "power": 1}
    if t == 1:
        return [dict(row, power=2 ** m) for m in range(int(spec.get("n_features", 1)))]
    if t in (3, 9) and row["lambda"] not in (-1.0, 1.0):
        raise ValueError(f"lambda must be +1 or -1: {spec}")
    return [row]


_PARAMS = ("type", "cutoff", "column", "eta", "rs", "lambda", "zeta", "theta_s", "power")


class AtomCenteredSymmetryFunctions(nn.Module):
    def __init__(self, species: Sequence, cutoffs: Sequence[dict], functions: Sequence[dict], mode: str = "none",
                 scale_range: Sequence[float] = (0.0, 1.0)):
        super().__init__()
        self.species = [_as_z(z) for z in species]
        if len(set(self.species)) != len(self.species):
            raise ValueError(f"repeated species in {self.species}")
        self.cutoffs = [_cutoff_spec(c) for c in cutoffs]
        if not self.cutoffs:
            raise ValueError("at least one cutoff function is needed")
        rows = [r for f in functions for r in _function_rows(f, len(self.cutoffs))]
        for r in rows:
            if r["element"] not in self.species or any(z not in self.species for z in r["neighbors"]):
                raise ValueError(f"symmetry function {r} names an element outside {self.species}")
        sp = {z: i for i, z in enumerate(self.species)}
        cols = {z: 0 for z in self.species}
        for r in rows:
            r["column"] = cols[r["element"]]
            cols[r["element"]] += 1
        self.functions = rows
        self.n_features = dict(cols)
        self._dim = max(cols.values()) if rows else 0
        self.cutoff = max(c["r_cut"] for c in self.cutoffs)
        if mode not in SCALING_MODES:
            raise ValueError(f"unknown scaling mode {mode!r}; choose one of {SCALING_MODES}")
        self.mode = mode
        self.scale_range = (float(scale_range[0]), float(scale_range[1]))
        n_sp = len(self.species)
        z2i = torch.full((119,), -1, dtype=torch.long)
        for z, i in sp.items():
            z2i[z] = i
        self.register_buffer("_z2i", z2i, persistent=False)
        valid = torch.zeros(n_sp, self._dim, dtype=torch.bool)
        for z, n in cols.items():
            valid[sp[z], :n] = True
        self.register_buffer("_valid", valid, persistent=False)
        table = torch.tensor([[float(r[k]) for k in _PARAMS] for r in rows] or [[0.0] * len(_PARAMS)],
                             dtype=torch.float64)
        for k, name in enumerate(_PARAMS):
            col = table[:, k]
            self.register_buffer(f"_p_{name}", col.long() if name in ("type", "cutoff", "column") else col.clone(),
                                 persistent=False)
        rad = [i for i, r in enumerate(rows) if r["type"] in (1, 2)]
        ang = [i for i, r in enumerate(rows) if r["type"] in (3, 8, 9)]
        self.register_buffer("_rad_lookup", self._lookup(rad, sp, 1), persistent=False)
        self.register_buffer("_ang_lookup", self._lookup(ang, sp, 2), persistent=False)
        self._ang_cutoff = max((self.cutoffs[rows[i]["cutoff"]]["r_cut"] for i in ang), default=0.0)
        self.register_buffer("stat_min", torch.zeros(n_sp, self._dim))
        self.register_buffer("stat_max", torch.ones(n_sp, self._dim))
        self.register_buffer("stat_avg", torch.zeros(n_sp, self._dim))

    def _lookup(self, idx: List[int], sp: dict, order: int) -> Tensor:
        """Function rows per (centre, neighbour species...), padded with -1."""
        n_sp = len(self.species)
        buckets: dict = {}
        for i in idx:
            r = self.functions[i]
            nb = [sp[z] for z in r["neighbors"]]
            keys = {(sp[r["element"]], *nb)}
            if order == 2:
                keys.add((sp[r["element"]], nb[1], nb[0]))
            for key in keys:
                buckets.setdefault(key, []).append(i)
        width = max((len(v) for v in buckets.values()), default=0)
        out = torch.full((n_sp,) * (order + 1) + (max(width, 1),), -1, dtype=torch.long)
        for key, rs in buckets.items():
            out[key + (slice(0, len(rs)),)] = torch.tensor(rs)
        return out[..., :width]

    @property
    def output_dim(self) -> int:
        return self._dim

    def _cutoff_values(self, r: Tensor) -> Tensor:
        return torch.stack([cutoff_function(r, c["kind"], c["r_cut"], c["r_inner"], c["exponent"])
                            for c in self.cutoffs], -1)

    def raw(self, data) -> Tensor:
        return self.compute_raw(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.num_nodes)

    def compute_raw(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor, n: int) -> Tensor:
        dtype, dev = edge_vec.dtype, edge_vec.device
        out = torch.zeros(n * max(self._dim, 1), dtype=dtype, device=dev)
        if self._dim == 0:
            return out.reshape(n, 0)
        sp = self._z2i[atomic_numbers]
        src, dst = edge_index[0], edge_index[1]
        r = torch.linalg.norm(edge_vec, dim=-1)
        if self._rad_lookup.shape[-1] > 0:
            out = out + self._radial(r, sp, src, dst, n)
        if self._ang_lookup.shape[-1] > 0:
            near = torch.nonzero(r < self._ang_cutoff).flatten()
            a, b = build_center_pairs(dst.index_select(0, near), n)
            if a.numel():
                out = out + self._angular(edge_vec, r, sp, src, dst, near.index_select(0, a), near.index_select(0, b), n)
        return out.reshape(n, self._dim)

    def _radial(self, r: Tensor, sp: Tensor, src: Tensor, dst: Tensor, n: int) -> Tensor:
        dt = r.dtype
        rows = self._rad_lookup[sp[dst].clamp(min=0), sp[src].clamp(min=0)]
        ok = (rows >= 0) & (sp[dst] >= 0).unsqueeze(-1) & (sp[src] >= 0).unsqueeze(-1)
        rows = rows.clamp(min=0)
        f = torch.gather(self._cutoff_values(r), 1, self._p_cutoff[rows])
        g2 = torch.exp(-self._p_eta.to(dt)[rows] * (r.unsqueeze(-1) - self._p_rs.to(dt)[rows]) ** 2) * f
        g1 = torch.pow(f, self._p_power.to(dt)[rows])
        val = torch.where(self._p_type[rows] == 1, g1, g2)
        val = torch.where(ok, val, torch.zeros_like(val))
        index = dst.unsqueeze(-1) * self._dim + self._p_column[rows]
        return torch.zeros(n * self._dim, dtype=dt, device=r.device).index_add(0, index.reshape(-1), val.reshape(-1))

    def _angular(self, vec: Tensor, r: Tensor, sp: Tensor, src: Tensor, dst: Tensor, e1: Tensor, e2: Tensor,
                 n: int) -> Tensor:
        dt = vec.dtype
        center = dst.index_select(0, e1)
        v1, v2 = vec.index_select(0, e1), vec.index_select(0, e2)
        r1, r2 = r.index_select(0, e1), r.index_select(0, e2)
        r3 = torch.linalg.norm(v1 - v2, dim=-1)
        cos = (v1 * v2).sum(-1) / (r1 * r2)
        s_c, s_1, s_2 = sp[center], sp[src.index_select(0, e1)], sp[src.index_select(0, e2)]
        rows = self._ang_lookup[s_c.clamp(min=0), s_1.clamp(min=0), s_2.clamp(min=0)]
        ok = (rows >= 0) & ((s_c >= 0) & (s_1 >= 0) & (s_2 >= 0)).unsqueeze(-1)
        rows = rows.clamp(min=0)
        fc1, fc2, fc3 = self._cutoff_values(r1), self._cutoff_values(r2), self._cutoff_values(r3)
        cut = self._p_cutoff[rows]
        f12 = torch.gather(fc1 * fc2, 1, cut)
        f123 = f12 * torch.gather(fc3, 1, cut)
        typ = self._p_type[rows]
        eta, zeta = self._p_eta.to(dt)[rows], self._p_zeta.to(dt)[rows]
        lam = self._p_lambda.to(dt)[rows]
        c = cos.unsqueeze(-1)
        base = (1.0 + lam * c).clamp(min=0.0)
        rsq = (r1 * r1 + r2 * r2).unsqueeze(-1)
        third = (r3 * r3).unsqueeze(-1)
        g3 = torch.pow(2.0, 1.0 - zeta) * torch.pow(base, zeta) * torch.where(
            typ == 3, torch.exp(-eta * (rsq + third)) * f123, torch.exp(-eta * rsq) * f12)
        m = _acos_margin(dt)
        theta = torch.rad2deg(torch.acos(cos.clamp(-1.0 + m, 1.0 - m))).unsqueeze(-1)
        ts = self._p_theta_s.to(dt)[rows]
        g8 = (torch.exp(-eta * (theta - ts) ** 2) + torch.exp(-eta * (theta - (360.0 - ts)) ** 2)
              + torch.exp(-eta * (theta + ts) ** 2) + torch.exp(-eta * (theta - (360.0 + ts)) ** 2)) * f123
        val = torch.where(typ == 8, g8, g3)
        val = torch.where(ok, val, torch.zeros_like(val))
        index = center.unsqueeze(-1) * self._dim + self._p_column[rows]
        return torch.zeros(n * self._dim, dtype=dt, device=vec.device).index_add(0, index.reshape(-1), val.reshape(-1))

    def scaling(self) -> Tuple[Tensor, Tensor]:
        """``(shift, factor)`` of ``G' = (G - shift) factor`` per element and function."""
        span = self.stat_max - self.stat_min
        flat = span == 0
        inv = torch.where(flat, torch.ones_like(span), 1.0 / torch.where(flat, torch.ones_like(span), span))
        if self.mode == "none":
            return torch.zeros_like(span), torch.ones_like(span)
        if self.mode == "scale":
            return self.stat_min, inv
        if self.mode == "center":
            return self.stat_avg, torch.ones_like(span)
        if self.mode == "center_scale":
            return self.stat_avg, inv
        smin, smax = self.scale_range
        factor = (smax - smin) * inv
        return self.stat_min - smin / factor, factor

    def scale(self, g: Tensor, atomic_numbers: Tensor) -> Tensor:
        if self.mode == "none":
            return g
        sp = self._z2i[atomic_numbers].clamp(min=0)
        shift, factor = self.scaling()
        scaled = (g - shift.to(g.dtype)[sp]) * factor.to(g.dtype)[sp]
        return torch.where(self._valid[sp], scaled, torch.zeros_like(scaled))

    def forward(self, data) -> Tensor:
        return self.compute(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.num_nodes)

    def compute(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor, num_nodes: int) -> Tensor:
        return self.scale(self.compute_raw(atomic_numbers, edge_index, edge_vec, num_nodes), atomic_numbers)

    @torch.no_grad()
    def fit_scaling(self, graphs: Iterable, mode: Optional[str] = None) -> None:
        """``stat_min``, ``stat_max`` and ``stat_avg`` from the atoms of ``graphs``."""
        if mode is not None:
            if mode not in SCALING_MODES:
                raise ValueError(f"unknown scaling mode {mode!r}")
            self.mode = mode
        n_sp = len(self.species)
        # running per-element statistics with scatter reductions over all atoms of a graph at
        # once: minimum and maximum by scatter_reduce, sums and counts by index_add
        lo = torch.full((n_sp, self._dim), math.inf, dtype=torch.float64)
        hi = torch.full((n_sp, self._dim), -math.inf, dtype=torch.float64)
        total = torch.zeros(n_sp, self._dim, dtype=torch.float64)
        count = torch.zeros(n_sp, dtype=torch.float64)
        z2i = self._z2i.cpu()
        for data in graphs:
            g = self.raw(data).detach().double().cpu()
            sp = z2i[data.atomic_numbers.cpu()]
            keep = sp >= 0
            g, sp = g[keep], sp[keep]
            idx = sp[:, None].expand_as(g)
            lo.scatter_reduce_(0, idx, g, "amin")
            hi.scatter_reduce_(0, idx, g, "amax")
            total.index_add_(0, sp, g)
            count.index_add_(0, sp, torch.ones_like(sp, dtype=torch.float64))
        missing = [self.species[i] for i in range(n_sp) if count[i] == 0]
        if missing:
            raise ValueError(f"no atoms of elements {missing} to compute the scaling from")
        valid = self._valid.cpu()
        dt = self.stat_min.dtype
        self.stat_min.copy_(torch.where(valid, lo, torch.zeros_like(lo)).to(dt))
        self.stat_max.copy_(torch.where(valid, hi, torch.ones_like(hi)).to(dt))
        self.stat_avg.copy_(torch.where(valid, total / count.clamp(min=1)[:, None], torch.zeros_like(total)).to(dt))
