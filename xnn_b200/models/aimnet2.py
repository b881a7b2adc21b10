"""AIMNet2 (Anstine, Zubatyuk & Isayev, Chem. Sci. 16, 10228, 2025).

``U = U_local + U_coul`` (D3 is added by the dispersion wrapper): Gaussian shells
``g_ijs = exp(-eta (r - r_s)^2) f_c(r)`` on ``[rbf_start, cutoff)``; a per-element embedding
with one value per channel and shell; the shell convolution of a per-atom quantity ``a_jcs``:
scalar sums ``sum_j g_ijs a_jcs`` and vector norms ``| sum_s w_csh sum_j g_ijs u_ij a_jcs |^2``;
message passes whose MLPs update the embedding and the charges (with neural charge equilibration
``q + f / sum f (Q - sum q)``, weights ``f^2``), the last giving the AIM vector; an energy MLP with
float64 per-element shifts; the short-range Coulomb energy removed under a mollifier (or cosine)
envelope and the Coulomb energy of the charges added back (all pairs, DSF, Ewald or PME). Two
charge channels (NSE) carry ``(Q +- (M - 1)) / 2``. Options, defaults and parameter names follow
the reference (``src/xnn/gnn/models/aimnet2.py``) so that the published checkpoints transplant.

The shell sums run as one edge-chunked contraction: gather ``a_src``, multiply with the edge's
``[g, g u]`` and scatter onto the centre (no padded neighbour matrix).
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.cutoff import CosineCutoff, MollifierCutoff
from ..nn.radial import GaussianRBF
from ..ops.scatter import refresh_ghosts, scatter_sum, structure_sum, whole_structure_sum
from .base import GNNPotential
from .electrostatics import COULOMB_CONSTANT, coulomb_direct, coulomb_dsf, coulomb_ewald, coulomb_pme, \
    ewald_parameters
from .registry import register_model

COULOMB_METHODS = ("simple", "dsf", "ewald", "pme", None)
LONG_RANGE_METHODS = ("dsf", "ewald", "pme")
SR_ENVELOPES = {"exp": MollifierCutoff, "cosine": CosineCutoff}
NQE_EPSILON = 1e-6
EDGE_CHUNK = 1 << 20


def _mlp(sizes: Sequence[int], final_activation: bool) -> nn.Sequential:
    layers = []
    for i in range(1, len(sizes)):
        lin = nn.Linear(sizes[i - 1], sizes[i])
        nn.init.xavier_normal_(lin.weight)
        nn.init.zeros_(lin.bias)
        layers.append(lin)
        if i < len(sizes) - 1 or final_activation:
            layers.append(nn.GELU())
    return nn.Sequential(*layers)


def shell_sums(nodes: Tensor, gsv: Tensor, edge_index: Tensor, weight: Tensor):
    """Scalar shell sums ``(N, C, S)`` and vector norms ``(N, C, H)`` of ``nodes (N, C, S)`` over the
    edges ``src -> dst`` with ``gsv (E, S, 4)`` = ``[g, g u_x, g u_y, g u_z]``."""
    src, dst = edge_index[0], edge_index[1]
    n, c, s = nodes.shape
    sums = nodes.new_zeros(n, c, s, 4)
    for e0 in range(0, src.shape[0], EDGE_CHUNK):
        e1 = e0 + EDGE_CHUNK
        part = nodes.index_select(0, src[e0:e1])[..., None] * gsv[e0:e1, None, :, :]
        sums = sums.index_add(0, dst[e0:e1], part)
    mixed = torch.einsum("csh,ncsd->nchd", weight, sums[..., 1:])
    return sums[..., 0], mixed.square().sum(-1)


class ShellConvolution(nn.Module):
    def __init__(self, n_channels: int, n_shells: int, n_combinations: int):
        super().__init__()
        w = torch.randn(n_channels, n_shells, n_combinations)
        w = (w - w.mean(1, keepdim=True)) / w.std(1, keepdim=True)
        self.weight = nn.Parameter(w)
        self.n_channels, self.n_shells, self.n_combinations = n_channels, n_shells, n_combinations
        self.output_dim = n_channels * (n_shells + n_combinations)

    def forward(self, nodes: Tensor, g: Tensor, gu: Tensor, edge_index: Tensor) -> Tensor:
        scalar, norms = shell_sums(nodes, torch.cat([g.unsqueeze(-1), gu], -1), edge_index, self.weight)
        return torch.cat([scalar.flatten(1), norms.flatten(1)], -1)


@register_model("aimnet2")
class AIMNet2(GNNPotential):
    head_modules = ("readout", "atom_ref")
    refreshes_ghosts = True

    def __init__(self, species, cutoff: float = 5.0, n_features: int = 16, n_rbf: int = 16, rbf_start: float = 0.8,
                 gaussian_width: Optional[float] = None, hidden=None, n_passes: int = 3,
                 n_vector_combinations: int = 12, aim_size: int = 256, readout_hidden=(128, 128),
                 charge_channels: int = 1, coulomb: Optional[str] = "simple", coulomb_sr_cutoff: float = 4.6,
                 coulomb_sr_envelope: str = "exp", lr_cutoff: float = 15.0, dsf_alpha: float = 0.2,
                 ewald_accuracy: float = 1e-6, pme_spline_order: int = 4, atomic_energies=None):
        super().__init__(species, cutoff)
        if hidden is None:
            if n_passes < 2:
                raise ValueError("AIMNet2 needs at least two passes (charges, then AIM)")
            hidden = [[512, 380]] * (n_passes - 1) + [[512, 380, 380]]
        hidden = [list(h) for h in hidden]
        if len(hidden) < 2:
            raise ValueError("AIMNet2 needs at least two passes (charges, then AIM)")
        if charge_channels not in (1, 2):
            raise ValueError("charge_channels must be 1 (closed shell) or 2 (NSE)")
        if coulomb not in COULOMB_METHODS:
            raise ValueError(f"coulomb must be one of {COULOMB_METHODS}, got {coulomb!r}")
        if coulomb_sr_envelope not in SR_ENVELOPES:
            raise ValueError(f"coulomb_sr_envelope must be one of {sorted(SR_ENVELOPES)}")
        if not 0.0 < float(ewald_accuracy) < 1.0:
            raise ValueError(f"ewald_accuracy must lie in (0, 1), got {ewald_accuracy}")
        if int(pme_spline_order) < 3:
            raise ValueError(f"pme_spline_order must be at least 3, got {pme_spline_order}")
        self.aev_cutoff = float(cutoff)
        self.n_features, self.n_rbf, self.charge_channels = int(n_features), int(n_rbf), int(charge_channels)
        self.aim_size = self.node_feature_dim = int(aim_size)
        self.coulomb = coulomb
        self.coulomb_sr_cutoff, self.lr_cutoff, self.dsf_alpha = float(coulomb_sr_cutoff), float(lr_cutoff), float(
            dsf_alpha)
        self.ewald_accuracy, self.pme_spline_order = float(ewald_accuracy), int(pme_spline_order)
        self.ewald_alpha, self.ewald_k_cutoff = ewald_parameters(self.lr_cutoff, self.ewald_accuracy)
        self.coulomb_constant = COULOMB_CONSTANT
        self.cutoff = max(self.aev_cutoff, self.lr_cutoff) if coulomb in LONG_RANGE_METHODS else self.aev_cutoff
        if gaussian_width is None:
            gaussian_width = (n_rbf / (cutoff - rbf_start)) ** 2
        self.rbf = GaussianRBF(n_rbf, cutoff, start=rbf_start, gamma=gaussian_width, endpoint=False)
        self.envelope = CosineCutoff(cutoff)
        ns = len(self.species)
        embed = torch.empty(ns, n_features)
        nn.init.orthogonal_(embed) if ns > 1 else nn.init.normal_(embed)
        self.embedding = nn.Embedding(ns, n_features * n_rbf)
        with torch.no_grad():
            self.embedding.weight.copy_(embed.repeat_interleave(n_rbf, dim=1))
        self.conv_a = ShellConvolution(n_features, n_rbf, n_vector_combinations)
        self.conv_q = ShellConvolution(charge_channels, n_rbf, n_vector_combinations)
        n_embed = n_features * n_rbf
        in_first = n_embed + self.conv_a.output_dim
        in_rest = in_first + charge_channels + self.conv_q.output_dim
        n_update = n_embed + 2 * charge_channels
        passes = [_mlp([in_first, *hidden[0], n_update], False)]
        passes += [_mlp([in_rest, *w, n_update], True) for w in hidden[1:-1]]
        passes.append(_mlp([in_rest, *hidden[-1], aim_size], True))
        self.passes = nn.ModuleList(passes)
        self.readout = _mlp([aim_size, *readout_hidden, 1], False)
        self.sr_envelope = SR_ENVELOPES[coulomb_sr_envelope](self.coulomb_sr_cutoff)
        self.atom_ref = nn.Embedding(200, 1)
        nn.init.zeros_(self.atom_ref.weight)
        self.atom_ref.double()
        if atomic_energies is not None:
            self.set_atomic_energies(atomic_energies)

    def _apply(self, fn, recurse=True):
        exact = self.atom_ref.weight.data
        out = super()._apply(fn, recurse)
        w = self.atom_ref.weight
        if w.dtype != torch.float64:     # the shifts (O(1000 eV)) stay float64
            w.data = exact.to(device=w.device, dtype=torch.float64)
        return out

    def receptive_field(self) -> Optional[float]:
        return None if self.coulomb is not None else len(self.passes) * self.aev_cutoff

    def equilibrate(self, charges: Tensor, weights: Tensor, total: Tensor, batch: Tensor, num_graphs: int,
                    eps: float = NQE_EPSILON) -> Tensor:
        wsum = whole_structure_sum(weights, batch, num_graphs) + eps
        surplus = total - whole_structure_sum(charges, batch, num_graphs)
        return charges + weights / wsum[batch] * surplus[batch]

    def channel_totals(self, total_charge: Tensor, spin_multiplicity: Tensor) -> Tensor:
        if self.charge_channels == 1:
            return total_charge[:, None]
        half = 0.5 * (spin_multiplicity - 1.0)
        return torch.stack([0.5 * total_charge + half, 0.5 * total_charge - half], -1)

    def _coulomb_long_range(self, q, pos, cell, pbc, batch, num_graphs, edge_index, r):
        periodic = pbc.any(dim=1)[batch] if cell is not None and pbc is not None else torch.zeros_like(batch,
                                                                                                       dtype=torch.bool)
        if self.coulomb == "simple":
            if bool(periodic.any()):
                raise ValueError("coulomb='simple' sums every pair of a molecule; periodic structures need "
                                 "coulomb='dsf', 'ewald' or 'pme'")
            return coulomb_direct(q, pos, batch)
        if self.coulomb == "dsf":
            return coulomb_dsf(q, edge_index, r, self.dsf_alpha, self.lr_cutoff)
        node = torch.zeros(q.shape[0], dtype=torch.float64, device=q.device)
        if cell is not None and pbc is not None:
            for i in range(num_graphs):
                if not bool(pbc[i].any()):
                    continue
                if not bool(pbc[i].all()):
                    raise ValueError("coulomb='ewald'/'pme' need full periodicity; use coulomb='dsf' for slabs")
                mask = batch == i
                idx = mask.nonzero().flatten()
                on = mask[edge_index[0]]
                local = (torch.cumsum(mask.long(), 0) - 1)[edge_index[:, on]]
                if self.coulomb == "ewald":
                    part = coulomb_ewald(q[idx], pos[idx], cell[i], local, r[on], self.ewald_alpha, self.lr_cutoff,
                                         self.ewald_k_cutoff)
                else:
                    part = coulomb_pme(q[idx], pos[idx], cell[i], local, r[on], self.ewald_alpha, self.lr_cutoff,
                                       self.ewald_accuracy, self.pme_spline_order)
                node = node.index_add(0, idx, part)
        free = ~periodic
        if bool(free.any()):
            idx = free.nonzero().flatten()
            node = node.index_add(0, idx, coulomb_direct(q[idx], pos[idx], batch[idx]))
        return node

    def _evaluate(self, z, edge_index, edge_vec, pos, cell, pbc, batch, num_graphs, totals) -> dict:
        index = self.z_to_index[z]
        if bool((index < 0).any()):
            raise ValueError(f"elements {sorted(set(z[index < 0].tolist()))} are not among the model's species "
                             f"{self.species}")
        n = z.shape[0]
        r_all = torch.linalg.norm(edge_vec, dim=-1)
        if self.cutoff > self.aev_cutoff:
            keep = r_all < self.aev_cutoff
            e_loc, v_loc, r = edge_index[:, keep], edge_vec[keep], r_all[keep]
        else:
            e_loc, v_loc, r = edge_index, edge_vec, r_all
        g = self.rbf(r) * self.envelope(r)[:, None]
        unit = -v_loc / r[:, None]
        gsv = torch.cat([g.unsqueeze(-1), g[:, :, None] * unit[:, None, :]], -1)
        nf, nr, nc = self.n_features, self.n_rbf, self.charge_channels
        a = self.embedding(index).view(n, nf, nr)
        q = None
        aim = None
        last = len(self.passes) - 1
        for i, mlp in enumerate(self.passes):
            if q is None:
                nodes, weight = a, self.conv_a.weight
            else:
                nodes = torch.cat([a, q[:, :, None].expand(-1, -1, nr)], 1)
                weight = torch.cat([self.conv_a.weight, self.conv_q.weight], 0)
            scalar, norms = shell_sums(nodes, gsv, e_loc, weight)
            if q is None:
                parts = [a.flatten(1), scalar.flatten(1), norms.flatten(1)]
            else:
                parts = [a.flatten(1), scalar[:, :nf].flatten(1), norms[:, :nf].flatten(1), q,
                         scalar[:, nf:].flatten(1), norms[:, nf:].flatten(1)]
            out = mlp(torch.cat(parts, -1))
            if i == last:
                aim = out
            else:
                dq, f, da = out.split([nc, nc, nf * nr], -1)
                q = refresh_ghosts(self.equilibrate(dq if q is None else q + dq, f.square(), totals, batch, num_graphs))
                a = refresh_ghosts(a + da.view(n, nf, nr))
        charges = q.sum(-1)
        node = self.readout(aim).squeeze(-1).to(torch.float64) + self.atom_ref(z).squeeze(-1)
        coul = torch.zeros_like(node)
        if self.coulomb is not None:
            src, dst = e_loc[0], e_loc[1]
            pair = 0.5 * self.coulomb_constant * self.sr_envelope(r) * charges[src] * charges[dst] / r
            coul = -scatter_sum(pair.to(torch.float64), dst, n)
            coul = coul + self._coulomb_long_range(charges, pos, cell, pbc, batch, num_graphs, edge_index, r_all)
            node = node + coul
        out = {"node_energy": node, "node_coulomb": coul, "node_features": aim, "charges": charges}
        if nc == 2:
            out["spin_charges"] = q[:, 0] - q[:, 1]
        return out

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        if self.coulomb is not None:
            raise RuntimeError("AIMNet2 with a Coulomb term needs whole structures (positions and net charge)")
        n = atomic_numbers.shape[0]
        dt = self.embedding.weight.dtype
        out = self._evaluate(atomic_numbers, edge_index, edge_vec, edge_vec.new_zeros(n, 3), None, None,
                             torch.zeros(n, dtype=torch.long, device=edge_vec.device), 1,
                             self.channel_totals(torch.zeros(1, dtype=dt, device=edge_vec.device),
                                                 torch.ones(1, dtype=dt, device=edge_vec.device)))
        return out["node_features"], out["node_energy"]

    def forward(self, data: AtomicGraph) -> dict:
        dt = self.embedding.weight.dtype
        b = data.num_graphs
        qt = data.total_charge.to(dt) if data.total_charge is not None else torch.zeros(b, dtype=dt, device=data.pos.device)
        m = (data.spin_multiplicity.to(dt) if data.spin_multiplicity is not None
             else torch.ones(b, dtype=dt, device=data.pos.device))
        out = self._evaluate(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.pos, data.cell, data.pbc,
                             data.batch, b, self.channel_totals(qt, m))
        q = out["charges"]
        res = {"node_energy": out["node_energy"], "energy": self.aggregate_energy(out["node_energy"], data),
               "node_features": out["node_features"], "charges": q,
               "dipole": scatter_sum(q[:, None] * data.pos.to(dt), data.batch, b),
               "energy_coulomb": structure_sum(out["node_coulomb"], data.batch, b)}
        if "spin_charges" in out:
            res["spin_charges"] = out["spin_charges"]
        return res

    @classmethod
    def from_config(cls, cfg) -> "AIMNet2":
        import ast
        e = dict(cfg.extra or {})
        seq = lambda v: ast.literal_eval(v) if isinstance(v, str) else v  # noqa: E731
        species = [int(z) for z in e.get("species") or [1, 6, 7, 8]]
        ae = e.get("atomic_energies")
        if isinstance(ae, dict):
            ae = [float(ae.get(z, ae.get(str(z), 0.0))) for z in species]
        return cls(species=species, cutoff=cfg.cutoff, n_features=cfg.n_features, n_rbf=cfg.n_rbf,
                   rbf_start=float(e.get("rbf_start", 0.8)), gaussian_width=e.get("gaussian_width"),
                   hidden=seq(e.get("hidden")), n_passes=int(cfg.n_interactions),
                   n_vector_combinations=int(e.get("n_vector_combinations", 12)), aim_size=int(e.get("aim_size", 256)),
                   readout_hidden=seq(e.get("readout_hidden", (128, 128))),
                   charge_channels=int(e.get("charge_channels", 1)), coulomb=e.get("coulomb", "simple"),
                   coulomb_sr_cutoff=float(e.get("coulomb_sr_cutoff", 4.6)),
                   coulomb_sr_envelope=e.get("coulomb_sr_envelope", "exp"), lr_cutoff=float(e.get("lr_cutoff", 15.0)),
                   dsf_alpha=float(e.get("dsf_alpha", 0.2)), ewald_accuracy=float(e.get("ewald_accuracy", 1e-6)),
                   pme_spline_order=int(e.get("pme_spline_order", 4)), atomic_energies=ae)
