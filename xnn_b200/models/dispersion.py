"""Dispersion corrections as potentials: shared pieces of the D3 (and D4) terms.

Behaviour follows the reference's ``src/xnn/common/models/dispersion.py``
(``DispersionCorrection`` at ``:667``, ``evaluate_on_graph`` at ``:844``, the switching
function, Gaussian reference weights and Axilrod-Teller-Muto term at ``:42-230``): a dispersion
term is evaluated on the neighbour list of the wrapper's cutoff (the larger of the model's and
the term's), the wrapped model sees only the edges within its own cutoff, and the energies add.

Reference data: the D3/D4 terms read Grimme's published reference tables (C6 references,
reference coordination numbers, radii) from ``.npz`` files that are not redistributed with this
package. :func:`reference_file` looks for them in ``$XNN_B200_DISPERSION_DATA`` and then in an
installed copy of the reference framework (its ``xnn/common/models/<name>``).
"""
from __future__ import annotations

import glob
import math
import os
from dataclasses import replace
from typing import Dict, Optional, Sequence

import numpy as np
import torch
from torch import Tensor, nn

from ..data.atomic_graph import AtomicGraph
from ..ops.scatter import build_triplets, scatter_sum, structure_sum
from .base import InteratomicPotential

#: CODATA 2018: Bohr radius in Angstrom and Hartree energy in eV
BOHR = 0.529177210903
HARTREE = 27.211386245988


def reference_file(name: str) -> str:
    """Path of a dispersion reference-data file (see module notes)."""
    cands = []
    env = os.environ.get("XNN_B200_DISPERSION_DATA")
    if env:
        cands.append(os.path.join(env, name))
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    cands.append(os.path.join(root, "baseline", "_ref", "xnn", "common", "models", name))
    cands += glob.glob(os.path.join(root, "baseline", "*", "xnn", "common", "models", name))
    for c in cands:
        if os.path.isfile(c):
            return c
    raise FileNotFoundError(
        f"dispersion reference data {name!r} not found; set XNN_B200_DISPERSION_DATA to a directory "
        "holding it (the published Grimme reference tables are not shipped with xnn_b200)")


def load_tables(name: str) -> Dict[str, np.ndarray]:
    with np.load(reference_file(name)) as d:
        return {k: d[k] for k in d.files}


def switching_function(r: Tensor, cutoff: float, width: float) -> Tensor:
    """Quintic window: 1 below ``cutoff - width``, 0 above ``cutoff`` (``width <= 0``: sharp)."""
    if width <= 0.0:
        return torch.ones_like(r)
    w = min(width, cutoff)
    x = torch.clamp((cutoff - r) / w, 0.0, 1.0)
    return x ** 3 * (10.0 + x * (6.0 * x - 15.0))


def gaussian_reference_weights(cn: Tensor, refcn: Tensor, valid: Tensor, wf: float,
                               ngw: Optional[Tensor] = None, eps_norm: float = 0.0,
                               n_gauss: Optional[int] = None) -> Tensor:
    """Normalised Gaussian weights ``(N, R)`` of the reference systems in the coordination number;
    when every Gaussian underflows the reference(s) with the largest CN take weight one.
    ``n_gauss``: the largest entry of ``ngw`` when the caller knows it (no device read-back)."""
    d2 = (cn[:, None] - refcn) ** 2
    if ngw is None:
        gw = torch.exp(-wf * d2)
    else:
        n_max = int(ngw.max()) if n_gauss is None else int(n_gauss)
        j = torch.arange(1, n_max + 1, device=cn.device)
        g = torch.exp(-wf * j.to(cn.dtype)[None, None, :] * d2[:, :, None])
        gw = torch.where(j[None, None, :] <= ngw[:, :, None], g, 0.0).sum(-1)
    gw = torch.where(valid, gw, 0.0)
    norm = gw.sum(1)
    ok = norm > eps_norm
    w = gw / torch.where(ok, norm, 1.0)[:, None]
    top = torch.where(valid, refcn, -math.inf).max(1).values
    fallback = (valid & ((refcn - top[:, None]).abs() < 1e-12)).to(cn.dtype)
    return torch.where(ok[:, None], w, fallback)


def three_body_energy(z: Tensor, edge_index: Tensor, edge_vec: Tensor, r: Tensor, c6_mat: Tensor,
                      r0_table: Tensor, s9: Tensor, alp3: float, cutoff: float, width: float, n_atoms: int,
                      chunk: int = 1 << 20) -> Tensor:
    """Per-atom Axilrod-Teller-Muto energy (hartree) with zero damping.

    Triples are pairs of edges sharing a centre, so a triangle is met once per corner; each
    visit assigns a third of the triangle's energy to its centre (the atom-resolved convention of
    the D3 codes, which also covers the self-image triangles of small periodic cells)."""
    e1, e2 = build_triplets(edge_index, n_atoms)
    once = e1 < e2                                  # unordered pairs of edges
    e1, e2 = e1[once], e2[once]
    center = edge_index[1][e1]
    out = torch.zeros(n_atoms, dtype=r.dtype, device=r.device)
    for s in range(0, e1.shape[0], chunk):
        a, b, c = e1[s:s + chunk], e2[s:s + chunk], center[s:s + chunk]
        j, k = edge_index[0][a], edge_index[0][b]
        v_a, v_b = edge_vec.index_select(0, a), edge_vec.index_select(0, b)
        ra, rb = r.index_select(0, a), r.index_select(0, b)
        raa, rbb = ra * ra, rb * rb
        v_jk = v_a - v_b
        rjk2 = (v_jk * v_jk).sum(-1)
        keep = (rjk2 <= cutoff * cutoff) & (rjk2 > 2.220446049250313e-16)
        rjk2 = torch.where(keep, rjk2, torch.ones_like(rjk2))
        rjk = torch.sqrt(rjk2)
        c9 = s9 * torch.sqrt((c6_mat[c, j] * c6_mat[c, k] * c6_mat[j, k]).abs())
        r0 = r0_table[z[c], z[j]] * r0_table[z[c], z[k]] * r0_table[z[j], z[k]]
        p2 = raa * rbb * rjk2
        p1 = torch.sqrt(p2)
        p3 = p2 * p1
        p5 = p3 * p2
        damp = 1.0 / (1.0 + 6.0 * (r0 / p1) ** alp3)
        ang = 0.375 * (raa + rjk2 - rbb) * (raa - rjk2 + rbb) * (-raa + rjk2 + rbb) / p5 + 1.0 / p3
        sw = (switching_function(ra, cutoff, width) * switching_function(rb, cutoff, width)
              * switching_function(rjk, cutoff, width))
        e = torch.where(keep, c9 * ang * damp * sw / 3.0, torch.zeros_like(p1))
        out = out + scatter_sum(e, c, n_atoms)
    return out


def atm_kernel_ok(vec: Tensor) -> bool:
    """Whether the three-body kernel (``csrc/dispersion.cu``) takes these edges."""
    if not (vec.is_cuda and vec.dtype == torch.float64):
        return False
    from .. import _ext
    return _ext.cuda_available() and hasattr(_ext.ops(), "atm")


class _ATMKernel(torch.autograd.Function):
    """Per-centre ATM energies from the kernel; the backward pass gives the edge-vector and C6-factor
    gradients for upstream gradients equal within each structure (a structure's energy)."""

    @staticmethod
    def forward(ctx, vec, fa, fb, ptr, center, nbr, z, r0, s9, alp3, cutoff, width, batch):
        from .. import _ext
        c6e = (fa.index_select(0, center) * fb.index_select(0, nbr)).sum(-1).contiguous()
        (e,) = _ext.ops().atm(ptr, nbr, vec.contiguous(), z, fa.contiguous(), fb.contiguous(), c6e, r0,
                              float(s9), float(alp3), float(cutoff), float(width), None)
        ctx.save_for_backward(vec, fa, fb, ptr, center, nbr, z, r0, c6e, batch)
        ctx.prm = (float(s9), float(alp3), float(cutoff), float(width))
        return e

    @staticmethod
    def backward(ctx, ge):
        from .. import _ext
        vec, fa, fb, ptr, center, nbr, z, r0, c6e, batch = ctx.saved_tensors
        ge = ge.contiguous().to(torch.float64)
        first = torch.zeros(int(batch.max()) + 1 if batch.numel() else 1, dtype=ge.dtype, device=ge.device)
        first = first.index_reduce_(0, batch, ge, "amax", include_self=False)
        if not torch.equal(first.index_select(0, batch), ge):
            raise NotImplementedError("the three-body kernel differentiates a structure's total energy "
                                      "(equal upstream gradients for the atoms of a structure)")
        gv, g6 = _ext.ops().atm(ptr, nbr, vec.contiguous(), z, fa.contiguous(), fb.contiguous(), c6e, r0,
                                *ctx.prm, ge)
        g_fa = torch.zeros_like(fa).index_add_(0, center, g6[:, None] * fb.index_select(0, nbr))
        g_fb = torch.zeros_like(fb).index_add_(0, nbr, g6[:, None] * fa.index_select(0, center))
        return (gv, g_fa, g_fb) + (None,) * 10


def three_body_energy_factored(z: Tensor, edge_index: Tensor, edge_vec: Tensor, fa: Tensor, fb: Tensor,
                               r0_table: Tensor, s9: float, alp3: float, cutoff: float, width: float,
                               batch: Tensor) -> Tensor:
    """:func:`three_body_energy` with ``C6_ij = fa_i . fb_j`` (D4's Casimir-Polder sums) on the
    kernel: one block per centre walking every pair of its edges (no triplet list in memory)."""
    n = z.shape[0]
    src, dst = edge_index
    order = torch.argsort(dst, stable=True)
    center, nbr = dst[order].contiguous(), src[order].contiguous()
    vec = edge_vec.index_select(0, order)
    ptr = torch.zeros(n + 1, dtype=torch.long, device=z.device)
    ptr[1:] = torch.cumsum(torch.bincount(dst, minlength=n), 0)
    return _ATMKernel.apply(vec, fa, fb, ptr, center, nbr, z.contiguous(), r0_table.contiguous(), s9, alp3, cutoff,
                            width, batch)


def evaluate_on_graph(term: nn.Module, data: AtomicGraph) -> Dict[str, Tensor]:
    """Run ``term.evaluate`` on a (batched) graph; adds ``"energy"`` ``(B,)``."""
    b = data.num_graphs
    dtype = data.compute_dtype or data.pos.dtype
    dev = data.pos.device
    pos = data.pos.to(dtype)
    cell = data.cell.to(dtype) if data.cell is not None else torch.zeros(b, 3, 3, dtype=dtype, device=dev)
    pbc = data.pbc if data.pbc is not None else torch.zeros(b, 3, dtype=torch.bool, device=dev)
    charge = data.total_charge if data.total_charge is not None else torch.zeros(b, dtype=dtype, device=dev)
    out = term.evaluate(data.atomic_numbers, pos, data.edge_index, data.edge_vectors().to(dtype), data.batch,
                        b, cell, pbc, charge.to(dtype))
    out["energy"] = structure_sum(out["node_energy"], data.batch, b)
    return out


class DispersionCorrection(InteratomicPotential):
    """A dispersion term standalone (``model=None``) or added to a short-range model.

    ``cutoff`` is ``max(model.cutoff, term.cutoff)``: build the graph with it. Outputs the
    combined ``"energy"`` / ``"node_energy"`` plus ``"energy_sr"``, ``"energy_disp"`` and the
    term's per-atom quantities."""

    _RENAME = {"charges": "eeq_charges"}

    def __init__(self, term: nn.Module, model: Optional[InteratomicPotential] = None):
        super().__init__()
        self.term = term
        self.model = model
        inner = float(getattr(model, "cutoff", 0.0)) if model is not None else 0.0
        self.cutoff = max(inner, float(term.cutoff))
        self.node_feature_dim = int(getattr(model, "node_feature_dim", 0)) if model is not None else int(
            term.n_features)

    def receptive_field(self) -> Optional[float]:
        inner = self.model.receptive_field() if self.model is not None else 0.0
        if inner is None:
            return None
        return max(float(inner), float(self.term.cutoff) * 2.0)

    def inner_graph(self, data: AtomicGraph) -> AtomicGraph:
        inner = float(getattr(self.model, "cutoff", self.cutoff))
        if inner >= self.cutoff:
            return data
        with torch.no_grad():
            keep = torch.linalg.norm(data.edge_vectors(), dim=-1) < inner
        return replace(data, edge_index=data.edge_index[:, keep], cell_shifts=data.cell_shifts[keep])

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        disp = evaluate_on_graph(self.term, data)
        node_disp, e_disp, feats = disp.pop("node_energy"), disp.pop("energy"), disp.pop("node_features")
        if self.model is None:
            out = {"node_energy": node_disp, "energy": e_disp, "node_features": feats,
                   "energy_sr": torch.zeros_like(e_disp)}
        else:
            out = dict(self.model(self.inner_graph(data)))
            out["energy_sr"] = out["energy"]
            out["energy"] = out["energy"] + e_disp.to(out["energy"].dtype)
            out["node_energy"] = out["node_energy"] + node_disp.to(out["node_energy"].dtype)
        out["energy_disp"] = e_disp
        for k, v in disp.items():
            out[self._RENAME.get(k, k)] = v
        return out


def options_from_extra(extra: dict, keys: Sequence[str]) -> dict:
    return {k: extra[k] for k in keys if k in extra}
