"""MACE energies on the fused ops (scalar hidden features), reading the reference modules' weights.

Per interaction, for ``C`` channels and spherical-harmonic degrees ``l <= lmax``:

* ``linear_up``: ``(N, C) @ W_up``; the species self-connection: one matrix per element;
* radial MLP: the folded e3nn layers as matrix products, the last one pre-scaled per
  degree by the tensor-product path coefficient;
* :func:`~xnn_b200.ops.mace_ops.conv`: messages summed into ``A (D, N, C)``;
* per-degree channel mixing ``A[l] @ W_l / avg_num_neighbors`` (one GEMM per degree on
  the component-major layout);
* :func:`~xnn_b200.ops.mace_ops.symmetric_contraction` with every order's weights
  concatenated, then the product linear and the residual.

The result equals the reference path of :class:`~xnn_b200.models.mace.MACE` to rounding.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
from torch import Tensor
from torch.nn import functional as F
from torch.utils.checkpoint import checkpoint

from ..ops import gemm
from ..ops import mace_ops as K
from ..ops import node_gemm as NG
from ..ops.lean_conv import lean_radial_conv
from ..ops.radial import radial_network
from ..ops.scatter import refresh_ghosts


def _linear_blocks(lin) -> List[Tensor]:
    """Scaled ``(mul_in, mul_out)`` matrices of an e3nn-layout Linear, in path order."""
    return lin.path_matrices()


def _species_weights(tp, n_el: int, block: int = 0) -> Tensor:
    """``(n_el, C_in, C_out)`` per-element matrices of one uvw path of a species tensor product."""
    ins = tp.instructions[block]
    off = sum(int(torch.tensor(i.path_shape).prod()) for i in tp.instructions[:block])
    c_in, ne, c_out = ins.path_shape
    from ..o3 import wigner_3j
    l = tp.irreps_out[ins.i_out].ir.l
    cg = float(wigner_3j(l, 0, l, dtype=torch.float64)[0, 0, 0]) if l == 0 else \
        float(wigner_3j(l, 0, l, dtype=torch.float64)[0, 0, 0])
    w = tp.weight[off:off + c_in * ne * c_out].view(c_in, ne, c_out)
    return (w * (ins.path_weight * cg)).permute(1, 0, 2)


def species_linear(h: Tensor, z: Tensor, Wz: Tensor, grouped: bool = False) -> Tensor:
    """``out[i] = h[i] @ Wz[z_i]`` for ``h (..., N, C_in)`` and ``Wz (n_el, C_in, C_out)``. With
    ``grouped`` (evaluation: constant weights) the rows of each element are multiplied by that
    element's matrix only, in one grouped tensor-core launch; otherwise by all matrices, keeping
    the matching block (differentiable in the weights)."""
    if grouped and NG.grouped_species_ok(h, Wz):
        return NG.species_linear(h, z, Wz)
    n_el, c_in, c_out = Wz.shape
    full = gemm.matmul(h, Wz.permute(1, 0, 2).reshape(c_in, n_el * c_out))   # (..., N, n_el*C_out)
    full = full.view(*h.shape[:-1], n_el, c_out)
    idx = z.view(*([1] * (h.dim() - 2)), -1, 1, 1).expand(*h.shape[:-1], 1, c_out)
    return full.gather(-2, idx).squeeze(-2)


def radial_mlp(net, rad: Tensor, col_scale: Optional[Tensor] = None) -> Tensor:
    layers = net.folded()
    h = rad
    for i, (W, fac, act, const) in enumerate(layers):
        last = i == len(layers) - 1
        w = W * fac
        if last and col_scale is not None:
            w = w * col_scale
        h = h @ w
        if act is not None:
            h = act(h)
            if const != 1.0:
                h = h * const
    return h


def _conv_path_scale(blk, like: Tensor) -> Tensor:
    """Per output column of the radial net, the tensor product's path coefficient ``w * CG(0,l,l)``.

    Cached per device and dtype on the block (built outside any CUDA-graph capture).
    """
    cache = blk.__dict__.setdefault("_fast_consts", {})
    key = ("path_scale", like.device, like.dtype)
    if key not in cache:
        cache[key] = _conv_path_scale_build(blk).to(like)
    return cache[key]


def _conv_path_scale_build(blk) -> Tensor:
    from ..o3 import wigner_3j
    tp = blk.conv_tp
    C = tp.irreps_in1[0].mul
    scales = []
    for ins in tp.instructions:
        l = tp.irreps_in2[ins.i_in2].ir.l
        cg = float(wigner_3j(0, l, l, dtype=torch.float64)[0, 0, 0]) * (2 * l + 1) ** 0.5
        scales.append(torch.full((C,), ins.path_weight * cg / (2 * l + 1) ** 0.5, dtype=torch.float64))
    return torch.cat(scales)


def _messages(h_up: Tensor, r: Tensor, Y: Tensor, plan: K.EdgePlan, blk, ef, P: int, C: int) -> Tensor:
    """Radial network and message pass of one interaction over the edges of ``plan``."""
    R = radial_network(r, blk.conv_tp_weights, _conv_path_scale(blk, r), ef.rbf.freqs, ef.rbf.norm,
                       ef.cutoff, ef.envelope.p).view(-1, P, C)
    return K.conv(h_up, R, Y, plan)


def _edge_chunks(plan: K.EdgePlan, edge_index: Tensor, max_edges: Optional[int]):
    """Receiver-contiguous edge chunks of at most ``max_edges`` edges (``None``: no chunking).

    With edges sorted by receiver, a chunk is the edge range of a range of receivers, so its
    messages fill a contiguous block of node rows. On CUDA the chunks go to
    :func:`~xnn_b200.ops.lean_conv.lean_radial_conv` (per-edge tensors of one chunk alive at a
    time, recomputed in the backward); on the CPU each chunk runs under activation checkpointing.
    Returns ``[((e0, e1), (n0, n1), plan_of_chunk), ...]``.
    """
    if max_edges is None or plan.n_edges <= max_edges or plan.dst_perm is not None:
        return None
    ptr = plan.dst_ptr.cpu()
    bounds, n0 = [], 0
    N = plan.n_nodes
    while n0 < N:
        limit = int(ptr[n0]) + max_edges
        n1 = int(torch.searchsorted(ptr, torch.tensor(limit), right=True)) - 1
        n1 = min(max(n1, n0 + 1), N)
        bounds.append((n0, n1))
        n0 = n1
    out = []
    for n0, n1 in bounds:
        e0, e1 = int(ptr[n0]), int(ptr[n1])
        ei = torch.stack([edge_index[0, e0:e1], edge_index[1, e0:e1] - n0])
        out.append(((e0, e1), (n0, n1), K.EdgePlan.build(ei, n1 - n0, assume_dst_sorted=True, n_src=N,
                                                        senders=False)))
    return out


def fast_node_features_energy(model, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor,
                              plan: Optional[K.EdgePlan] = None) -> Tuple[Tensor, Tensor]:
    N = atomic_numbers.shape[0]
    z = model.z_to_index[atomic_numbers].clamp(min=0)
    e0 = model.atom_ref(atomic_numbers).squeeze(-1)
    if plan is None:
        plan = K.EdgePlan.build(edge_index, N)
    ef = model.edge_feat
    lmax = model.max_ell
    P = lmax + 1
    Y, _ = K.edge_geometry(edge_vec, lmax, ef.rbf.freqs, ef.rbf.norm, ef.cutoff, ef.envelope.p)
    r = torch.linalg.norm(edge_vec, dim=-1)
    chunks = _edge_chunks(plan, edge_index, getattr(model, "edge_chunk", None)) \
        if not model.training else None
    n_el = len(model.species)
    C = model.num_features
    grouped = not model.training
    emb = model.node_embedding
    h = _linear_blocks(emb)[0].index_select(0, z)                       # (N, C)
    inter = torch.zeros_like(e0)
    feats = []
    for t, (blk, prod, readout) in enumerate(zip(model.interactions, model.products, model.readouts)):
        if t > 0:
            h = refresh_ghosts(h)
        sc = species_linear(h, z, _species_weights(blk.skip_tp, n_el), grouped) if blk.residual else None
        h_up = gemm.matmul(h, _linear_blocks(blk.linear_up)[0])
        if chunks is None:
            A = _messages(h_up, r, Y, plan, blk, ef, P, C)               # (D, N, C)
        elif h_up.is_cuda:
            A = lean_radial_conv(h_up, r, Y, chunks, blk.conv_tp_weights, _conv_path_scale(blk, r),
                                 ef.rbf.freqs, ef.rbf.norm, ef.cutoff, ef.envelope.p, P, plan)
        else:
            A = torch.cat([checkpoint(_messages, h_up, r[e0:e1], Y[e0:e1], sub, blk, ef, P, C,
                                      use_reentrant=False) for (e0, e1), _, sub in chunks], dim=1)
        mats = _linear_blocks(blk.linear)
        # per-degree blocks as one split (its adjoint is one concatenation; slices would each
        # add a full-size zero-filled gradient)
        degrees = [2 * l + 1 for l in range(P)]
        parts = [gemm.matmul(blk_l, mats[l] / blk.avg_num_neighbors)
                 for l, blk_l in enumerate(A.split(degrees, 0))]
        A2 = torch.cat(parts, 0) if P > 1 else parts[0]
        if not blk.residual:
            Wl = [_species_weights(blk.skip_tp, n_el, l) for l in range(P)]
            if grouped and NG.grouped_species_ok(A2, Wl[0]):
                A2 = NG.species_linear_blocks(A2, z, Wl, degrees)       # every degree in one launch
            else:
                outs = [species_linear(blk_l, z, Wl[l], grouped) for l, blk_l in enumerate(A2.split(degrees, 0))]
                A2 = torch.cat(outs, 0) if P > 1 else outs[0]
        sym = prod.symmetric_contractions.contractions[0]
        W = torch.cat(list(sym.weights), dim=1)                         # (n_el, K, C)
        B = K.symmetric_contraction(A2, W, z, lmax, sym.correlation)
        h = gemm.matmul(B, _linear_blocks(prod.linear)[0])
        if prod.use_sc and sc is not None:
            h = h + sc
        inter = inter + readout(h).squeeze(-1)
        feats.append(h)
    node_energy = e0 + model.scale_shift(inter)
    return torch.cat(feats, dim=-1), node_energy
