"""Grimme D3 dispersion (zero, rational Becke-Johnson, modified-zero and optimized-power damping).

Written from Grimme, Antony, Ehrlich & Krieg, J. Chem. Phys. 132, 154104 (2010) and Grimme,
Ehrlich & Goerigk, J. Comput. Chem. 32, 1456 (2011), with the conventions of the reference's
``src/xnn/common/models/d3.py`` (``DFTD3`` at ``:483``): the exponential counting function
(k1 = 16, 4/3-scaled covalent radii, 40 bohr cutoff), Gaussian CN weights (k3 = 4) with the
highest-CN fallback, ``C6 = sum_ab W_a W_b C6ref``, ``C8 = 3 C6 sqrt(Q_A Q_B)`` from the
``<r4>/<r2>`` factors, the 60 / 40 bohr pair / triple cutoffs and the optional ATM term.
Inputs in Angstrom, energies in eV, atomic units inside. Reference data: the 2024 set of the
published tables (``d3_reference.npz``; see :mod:`xnn_b200.models.dispersion`).
"""
from __future__ import annotations

from typing import Dict, Optional

import numpy as np
import torch
from torch import Tensor, nn

from ..ops.scatter import scatter_sum, structure_sum
from .dispersion import (BOHR, HARTREE, DispersionCorrection, evaluate_on_graph, gaussian_reference_weights,
                         load_tables, options_from_extra, switching_function, three_body_energy)
from .registry import register_model

KCN, WF, RS9 = 16.0, 4.0, 4.0 / 3.0
MAX_Z = 103
CUTOFF_PAIR_AU, CUTOFF_TRIPLE_AU, CUTOFF_CN_AU = 60.0, 40.0, 40.0
DAMPINGS = ("bj", "zero", "mzero", "op")
#: published damping parameters (Grimme et al.) of a few functionals
PARAMS_BJ = {"pbe0": dict(s8=1.2177, a1=0.4145, a2=4.8593), "pbe": dict(s8=0.7875, a1=0.4289, a2=4.4407),
             "b3lyp": dict(s8=1.9889, a1=0.3981, a2=4.4211), "tpss": dict(s8=1.9435, a1=0.4535, a2=4.4752)}
PARAMS_ZERO = {"pbe0": dict(s8=0.928, rs6=1.287), "pbe": dict(s8=0.722, rs6=1.217),
               "b3lyp": dict(s8=1.703, rs6=1.261)}


class _TwoBodyKernel(torch.autograd.Function):
    """The two-body energy per atom on the native passes (``csrc/d3.cu``, OpenMP twin on the
    CPU) with analytic edge gradients. The backward scales them by the incoming gradient of the
    receiving atom, which is exact when that gradient is the same on both ends of every edge
    (energies of whole structures, the forces / stress / energy-loss case); first derivatives
    only."""

    @staticmethod
    def forward(ctx, vec, z, plan, tables, damping, prm):
        r = torch.linalg.norm(vec, dim=-1).contiguous()
        from .. import _ext
        e_atom, cn, g, w = _ext.ops().d3_two_body(z, plan.dst_ptr, plan.dst_perm if plan.dst_perm is not None
                                               else z.new_zeros(0), plan.src, plan.dst, r, vec.contiguous(),
                                               *tables, damping, prm, True)
        ctx.save_for_backward(g, plan.dst)
        ctx.mark_non_differentiable(cn, w)
        return e_atom, cn, w

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, ge, gcn, gw):
        g, dst = ctx.saved_tensors
        return g * ge.index_select(0, dst)[:, None], None, None, None, None, None


class DFTD3(nn.Module):
    """The D3 energy of one or several structures from a neighbour list (see module notes)."""

    def __init__(self, damping: str = "bj", s6: float = 1.0, s8: Optional[float] = None, s9: float = 0.0,
                 a1: float = 0.4145, a2: float = 4.8593, rs6: float = 1.287, rs8: float = 1.0, alp: float = 14.0,
                 bet: float = 0.0, cutoff_pair: float = CUTOFF_PAIR_AU * BOHR,
                 cutoff_triple: float = CUTOFF_TRIPLE_AU * BOHR, cutoff_cn: float = CUTOFF_CN_AU * BOHR,
                 switch_width_pair: float = 0.0, switch_width_triple: float = 0.0, trainable: bool = False,
                 references: str = "2024", **unused):
        super().__init__()
        damping = {"rational": "bj", "d3bj": "bj"}.get(damping.lower(), damping.lower())
        if damping not in DAMPINGS:
            raise ValueError(f"damping must be one of {DAMPINGS}, got {damping!r}")
        if str(references) != "2024":
            raise NotImplementedError("only the 2024 D3 reference set is built")
        self.damping = damping
        if s8 is None:
            s8 = PARAMS_BJ["pbe0"]["s8"] if damping in ("bj", "op") else PARAMS_ZERO["pbe0"]["s8"]
        self.alp = float(alp)
        self.cutoff_pair, self.cutoff_triple, self.cutoff_cn = float(cutoff_pair), float(cutoff_triple), float(cutoff_cn)
        self.cutoff = max(self.cutoff_pair, self.cutoff_triple, self.cutoff_cn)
        self.switch_width_pair, self.switch_width_triple = float(switch_width_pair), float(switch_width_triple)
        self.n_features = 2
        dt = torch.get_default_dtype()
        for name, v in [("s6", s6), ("s8", s8), ("s9", s9), ("a1", a1), ("a2", a2), ("rs6", rs6), ("rs8", rs8),
                        ("bet", bet)]:
            t = torch.tensor(float(v), dtype=dt)
            if trainable:
                setattr(self, name, nn.Parameter(t))
            else:
                self.register_buffer(name, t)
        tab = load_tables("d3_reference.npz")
        zz = np.arange(tab["r4r2_raw"].shape[0], dtype=np.float64)
        buf = lambda n, a, d=dt: self.register_buffer(n, torch.tensor(a, dtype=d), persistent=False)  # noqa: E731
        buf("rcov", 4.0 / 3.0 * tab["covalent_radius_aa"] / BOHR)
        buf("r4r2", np.sqrt(0.5 * tab["r4r2_raw"] * np.sqrt(zz)))
        buf("rvdw", tab["rvdw_aa"] / BOHR)
        buf("nref", tab["nref"], torch.long)
        buf("refcn", tab["refcn"])
        buf("c6ref", tab["c6"])

    # ------------------------------------------------------------------ pieces (atomic units)
    def coordination_numbers(self, z: Tensor, edge_index: Tensor, r: Tensor, n: int) -> Tensor:
        src, dst = edge_index[0], edge_index[1]
        rc = self.rcov[z[dst]] + self.rcov[z[src]]
        count = 1.0 / (1.0 + torch.exp(-KCN * (rc / r - 1.0)))
        return scatter_sum(torch.where(r <= self.cutoff_cn / BOHR, count, torch.zeros_like(count)), dst, n)

    def reference_weights(self, z: Tensor, cn: Tensor) -> Tensor:
        refcn = self.refcn[:, z].t()
        valid = torch.arange(refcn.shape[1], device=z.device)[None, :] < self.nref[z][:, None]
        return gaussian_reference_weights(cn, refcn, valid, WF)

    def species_vectors(self, z: Tensor, w: Tensor) -> Tensor:
        """``V[i, b, Z] = sum_a W_ia C6ref[a, b, Z_i, Z]`` ``(N, 7, Zmax + 1)``, one species at a time."""
        n_slots, n_z = self.refcn.shape
        v = torch.zeros((z.shape[0], n_slots, n_z), dtype=w.dtype, device=z.device)
        for zi in torch.unique(z).tolist():
            rows = torch.nonzero(z == zi).squeeze(1)
            v = v.index_put((rows,), torch.einsum("na,abz->nbz", w[rows], self.c6ref[:, :, zi, :]))
        return v

    def pair_c6(self, z: Tensor, w: Tensor, v: Tensor, i: Tensor, j: Tensor) -> Tensor:
        return (v[i, :, z[j]] * w[j]).sum(-1)

    def c6_matrix(self, z: Tensor, w: Tensor, v: Tensor) -> Tensor:
        return torch.einsum("jb,ibj->ij", w, v[:, :, z])

    def two_body_energy(self, z: Tensor, edge_index: Tensor, r: Tensor, c6: Tensor, n: int) -> Tensor:
        src, dst = edge_index[0], edge_index[1]
        zi, zj = z[dst], z[src]
        rr = 3.0 * self.r4r2[zi] * self.r4r2[zj]
        r0 = self.a1 * torch.sqrt(rr) + self.a2 if self.damping in ("bj", "op") else self.rvdw[zi, zj]
        r2 = r * r
        r6, r8 = r2 ** 3, r2 ** 4
        if self.damping == "bj":
            t6, t8 = 1.0 / (r6 + r0 ** 6), 1.0 / (r8 + r0 ** 8)
        elif self.damping == "zero":
            t6 = 1.0 / (1.0 + 6.0 * (self.rs6 * r0 / r) ** self.alp) / r6
            t8 = 1.0 / (1.0 + 6.0 * (self.rs8 * r0 / r) ** (self.alp + 2.0)) / r8
        elif self.damping == "mzero":
            t6 = 1.0 / (1.0 + 6.0 * (r / (self.rs6 * r0) + self.bet * r0) ** (-self.alp)) / r6
            t8 = 1.0 / (1.0 + 6.0 * (r / (self.rs8 * r0) + self.bet * r0) ** (-(self.alp + 2.0))) / r8
        else:
            rb, ab = r ** self.bet, r0 ** self.bet
            t6 = rb / (rb * r6 + ab * r0 ** 6)
            t8 = rb / (rb * r8 + ab * r0 ** 8)
        sw = switching_function(r, self.cutoff_pair / BOHR, self.switch_width_pair / BOHR)
        return scatter_sum(-0.5 * c6 * sw * (self.s6 * t6 + self.s8 * rr * t8), dst, n)

    # ------------------------------------------------------------------ native two-body path
    def kernels_usable(self, edge_vec: Tensor) -> bool:
        """The native passes take the two-body term: rational or zero damping, no three-body term,
        fixed parameters, evaluation mode (first derivatives), ``use_kernels`` not switched off."""
        from .. import _ext
        return (getattr(self, "use_kernels", True) and not self.training and self.damping in ("bj", "zero")
                and not any(isinstance(getattr(self, k), nn.Parameter) for k in ("s6", "s8", "a1", "a2"))
                and float(self.s9) == 0.0 and _ext.available() and hasattr(_ext.ops(), "d3_two_body"))

    def _tables(self, device):
        key = str(device)
        cache = self.__dict__.setdefault("_table_cache", {})
        if key not in cache:
            f = lambda t: t.detach().to(device=device, dtype=torch.float64).contiguous()  # noqa: E731
            cache[key] = (f(self.rcov), f(self.r4r2), f(self.rvdw), self.nref.to(device).contiguous(),
                          f(self.refcn), f(self.c6ref))
        return cache[key]

    def _two_body_kernel(self, z: Tensor, edge_index: Tensor, vec: Tensor):
        from ..ops.mace_ops import EdgePlan
        n = z.shape[0]
        plan = EdgePlan.build(edge_index, n)
        prm = [float(self.s6), float(self.s8), float(self.a1), float(self.a2), float(self.rs6), float(self.rs8),
               float(self.alp), KCN, WF, self.cutoff_cn / BOHR, self.cutoff_pair / BOHR, self.switch_width_pair / BOHR]
        return _TwoBodyKernel.apply(vec.to(torch.float64), z.contiguous(), plan, self._tables(z.device),
                                    0 if self.damping == "bj" else 1, prm)

    # ------------------------------------------------------------------ evaluation
    def evaluate(self, atomic_numbers: Tensor, pos: Tensor, edge_index: Tensor, edge_vec: Tensor, batch: Tensor,
                 num_graphs: int, cell: Tensor, pbc: Tensor, total_charge: Tensor) -> Dict[str, Tensor]:
        """Per-atom energy (eV), per-structure two/three-body energies, coordination numbers,
        dense C6 matrix (hartree bohr^6; empty above 20000 atoms) and features ``(N, 2)``."""
        z = atomic_numbers
        n = z.shape[0]
        if bool((z > MAX_Z).any()) or bool((z < 1).any()):
            raise ValueError("D3 reference data cover atomic numbers 1..103")
        vec = edge_vec / BOHR
        if self.kernels_usable(edge_vec):
            e2, cn, w = self._two_body_kernel(z, edge_index, vec)
            c6_self = torch.einsum("na,abn,nb->n", w, self._tables(z.device)[5][:, :, z, z], w)
            e2, cn, c6_self = (t.to(edge_vec.dtype) for t in (e2, cn, c6_self))
            empty = torch.zeros((0, 0), dtype=edge_vec.dtype, device=edge_vec.device)
            return {"node_energy": e2 * HARTREE,
                    "energy_2body": structure_sum(e2, batch, num_graphs) * HARTREE,
                    "energy_3body": torch.zeros(num_graphs, dtype=e2.dtype, device=e2.device),
                    "coordination_numbers": cn, "c6_matrix": empty,
                    "node_features": torch.stack([cn, c6_self], 1)}
        r = torch.linalg.norm(vec, dim=-1)
        cn = self.coordination_numbers(z, edge_index, r, n)
        w = self.reference_weights(z, cn)
        v = self.species_vectors(z, w)
        in_pair = r <= self.cutoff_pair / BOHR
        pidx = edge_index[:, in_pair]
        c6 = self.pair_c6(z, w, v, pidx[1], pidx[0])
        e2 = self.two_body_energy(z, pidx, r[in_pair], c6, n)
        e3 = torch.zeros_like(e2)
        dense = n <= 20000
        c6_mat = self.c6_matrix(z, w, v) if dense else torch.zeros((0, 0), dtype=r.dtype, device=r.device)
        if bool(self.s9 != 0.0):
            if not dense:
                raise ValueError("the D3 three-body term needs the dense C6 matrix (> 20000 atoms); set s9 = 0")
            m = r <= self.cutoff_triple / BOHR
            e3 = three_body_energy(z, edge_index[:, m], vec[m], r[m], c6_mat, RS9 * self.rvdw, self.s9,
                                   (self.alp + 2.0) / 3.0, self.cutoff_triple / BOHR,
                                   self.switch_width_triple / BOHR, n)
        c6_self = c6_mat.diagonal() if dense else self.pair_c6(z, w, v, torch.arange(n, device=z.device),
                                                                 torch.arange(n, device=z.device))
        return {"node_energy": (e2 + e3) * HARTREE,
                "energy_2body": structure_sum(e2, batch, num_graphs) * HARTREE,
                "energy_3body": structure_sum(e3, batch, num_graphs) * HARTREE,
                "coordination_numbers": cn, "c6_matrix": c6_mat,
                "node_features": torch.stack([cn, c6_self], 1)}

    def forward(self, data) -> Dict[str, Tensor]:
        return evaluate_on_graph(self, data)


D3_KEYS = ("damping", "s6", "s8", "s9", "a1", "a2", "rs6", "rs8", "alp", "bet", "references", "cutoff_pair",
           "cutoff_triple", "cutoff_cn", "switch_width_pair", "switch_width_triple", "trainable")


@register_model("d3")
class D3Dispersion(DispersionCorrection):
    """D3 as a potential: standalone, or added to ``model`` (``model.extra["dispersion"]``)."""

    def __init__(self, model=None, **d3_options):
        super().__init__(DFTD3(**d3_options), model)

    @property
    def d3(self) -> DFTD3:
        return self.term

    @classmethod
    def from_config(cls, cfg) -> "D3Dispersion":
        return cls(**options_from_extra(dict(getattr(cfg, "extra", {}) or {}), D3_KEYS))
