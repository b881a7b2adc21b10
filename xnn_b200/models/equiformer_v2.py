"""EquiformerV2 (Liao, Wood, Das and Smidt, ICLR 2024): equivariant graph attention whose
messages are SO(2) convolutions in per-edge frames.

Each edge's frame rotates its direction onto +y; node features (``(N, (lmax+1)^2, C)``, real
spherical-harmonic coefficients) of both ends are rotated by the block-diagonal Wigner matrices of
that frame with orders truncated to ``|m| <= mmax`` and reordered order-major, so that the
convolution is a dense linear map per order ``m`` (a complex product for ``m > 0``) weighted by a
radial MLP. Attention logits come from extra ``m = 0`` channels; the nonlinearity is a gate, a
point-wise SiLU on an S2 grid, or the separable form (SiLU on the scalars, the grid for the rest);
feed-forward blocks act per degree with an MLP on the grid. Norms: separable layer norm, per-degree
layer norm or RMS norm.

The edge frame (the minimal rotation taking the edge onto +y, ``diag(1, -1, -1)`` at the south
pole), the Wigner matrices by Clebsch-Gordan recursion from the 3x3 rotation, the order-major
layout, the ``sqrt((2l+1)/(2 mmax+1))`` rescaling of degrees above ``mmax``, parameter names and
initialisation follow the reference (``src/xnn/trfnn/models/equiformer_v2.py``) so state dicts
transplant and the roll of each frame about its axis (to which the grid activations are
sensitive) is the same.
"""
from __future__ import annotations

import math
from functools import lru_cache
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn import PolynomialCutoff
from ..nn.radial import GaussianRBF
from ..o3 import FromS2Grid, ToS2Grid, spherical_harmonics, wigner_3j
from ..ops.scatter import scatter_sum, segment_softmax
from .equiformer import GraphDropPath, RadialMLP, SmoothLeakyReLU
from .et import TransformerPotential
from .registry import register_model

AVG_NUM_NODES = 18.03065905448718
AVG_DEGREE = 15.57930850982666
ACTIVATIONS = ("sep_s2", "s2", "gate")
NORMS = ("layer_norm_sh", "layer_norm", "rms_norm_sh")


def _orders(lmax: int, mmax: int) -> List[int]:
    return [min(l, mmax) for l in range(lmax + 1)]


def reduced_index(lmax: int, mmax: int) -> List[int]:
    """Positions (in the full ``(lmax+1)^2`` layout) of the coefficients with ``|m| <= mmax``."""
    return [l * l + l + m for l, mm in enumerate(_orders(lmax, mmax)) for m in range(-mm, mm + 1)]


def m_primary_order(lmax: int, mmax: int) -> List[int]:
    """Permutation of the reduced degree-major layout into order-major: all ``m = 0``, then
    ``+m`` and ``-m`` for ``m = 1 .. mmax`` (degrees ascending within each)."""
    zero, at = [], 0
    for mm in _orders(lmax, mmax):
        zero.append(at + mm)
        at += 2 * mm + 1
    order = list(zero)
    for m in range(1, mmax + 1):
        order += [zero[l] + m for l in range(m, lmax + 1)] + [zero[l] - m for l in range(m, lmax + 1)]
    return order


def grid_resolution(lmax: int, mmax: int, resolution: Optional[int]) -> Tuple[int, int]:
    if resolution is not None:
        return int(resolution), int(resolution)
    return 2 * (lmax + 1), (2 * (mmax + 1) + 1 if lmax == mmax else 2 * mmax + 1)


def _rescale(lmax: int, mmax: int) -> List[float]:
    return [math.sqrt((2 * l + 1) / (2 * mmax + 1)) if l > mmax else 1.0 for l in range(lmax + 1)]


@lru_cache(maxsize=None)
def s2_grid_matrices(lmax: int, mmax: int, res_beta: int, res_alpha: int) -> Tuple[Tensor, Tensor]:
    """``(P, R)`` float64 synthesis and analysis matrices between the reduced coefficients and the
    ``P = res_beta * res_alpha`` grid values."""
    to = ToS2Grid(lmax, (res_beta, res_alpha), "component", dtype=torch.float64)
    fr = FromS2Grid((res_beta, res_alpha), lmax, "component", dtype=torch.float64)
    to_mat = torch.einsum("mbi,am->bai", to.shb, to.sha)
    from_mat = torch.einsum("am,mbi->bai", fr.sha, fr.shb)
    scale = torch.tensor([s for l, s in enumerate(_rescale(lmax, mmax)) for _ in range(2 * l + 1)], dtype=torch.float64)
    idx = torch.tensor(reduced_index(lmax, mmax))
    return ((to_mat * scale)[:, :, idx].reshape(res_beta * res_alpha, -1),
            (from_mat * scale)[:, :, idx].reshape(res_beta * res_alpha, -1))


class S2Grid(nn.Module):
    """Reduced coefficients ``(B, R, C)`` to grid values ``(P, B, C)`` and back."""

    def __init__(self, lmax: int, mmax: int, resolution: Optional[int] = None):
        super().__init__()
        to_mat, from_mat = s2_grid_matrices(lmax, mmax, *grid_resolution(lmax, mmax, resolution))
        self.register_buffer("to_grid_mat", to_mat, persistent=False)
        self.register_buffer("from_grid_mat", from_mat, persistent=False)

    def to_grid(self, x: Tensor) -> Tensor:
        b, r, c = x.shape
        m = self.to_grid_mat.to(x.dtype)
        return torch.mm(m, x.transpose(0, 1).reshape(r, b * c)).view(m.shape[0], b, c)

    def from_grid(self, y: Tensor) -> Tensor:
        p, b, c = y.shape
        m = self.from_grid_mat.to(y.dtype)
        return torch.mm(m.t(), y.reshape(p, b * c)).view(m.shape[1], b, c).transpose(0, 1)

    def forward(self, x: Tensor) -> Tensor:
        return self.from_grid(F.silu(self.to_grid(x)))


def edge_rotation(vec: Tensor) -> Tensor:
    """``(E, 3, 3)`` rotations taking each edge direction onto +y (the minimal rotation, about
    ``n x e_y``; ``diag(1, -1, -1)`` for a direction at -y)."""
    n = vec / torch.linalg.norm(vec, dim=-1, keepdim=True)
    x, y, z = n.unbind(-1)
    s2 = x * x + z * z
    tiny = 1e-20
    # 1 / (1 + y), written as (1 - y) / (x^2 + z^2) in the lower hemisphere to stay accurate
    k = torch.where(y >= 0, 1.0 / (1.0 + y.clamp(min=0.0)), (1.0 - y) / torch.where(s2 < tiny, torch.ones_like(s2), s2))
    rot = torch.stack([y + z * z * k, -x, -x * z * k, x, y, z, -x * z * k, -z, y + x * x * k], -1).reshape(-1, 3, 3)
    flip = torch.diag(vec.new_tensor([1.0, -1.0, -1.0]))
    return torch.where(((y < 0) & (s2 < tiny))[:, None, None], flip.expand_as(rot), rot)


class EdgeFrames(nn.Module):
    """Wigner matrices ``D^l`` (``l = 0 .. lmax``) of the edge frames: ``D^1`` is the rotation in
    the harmonics' axis order, ``D^l = C (D^{l-1} x D^1) C^T`` with the unitary coupling ``C`` of
    ``(l-1) x 1 -> l``."""

    def __init__(self, lmax: int):
        super().__init__()
        self.lmax = int(lmax)
        basis = spherical_harmonics(1, torch.eye(3, dtype=torch.float64), normalize=True, normalization="norm").T
        self.register_buffer("basis", basis.contiguous())
        blocks, starts = [], [0, 0, 0]
        for l in range(2, self.lmax + 1):
            c = wigner_3j(l - 1, 1, l, dtype=torch.float64).permute(2, 0, 1) * math.sqrt(2 * l + 1)
            blocks.append(c.reshape(-1))
            starts.append(starts[-1] + c.numel())
        self.cg_starts = starts
        self.register_buffer("cg", torch.cat(blocks) if blocks else torch.zeros(0, dtype=torch.float64))

    def forward(self, vec: Tensor) -> List[Tensor]:
        rot = edge_rotation(vec)
        basis = self.basis.to(rot.dtype)
        d1 = basis @ rot @ basis.t()
        out = [torch.ones_like(rot[:, :1, :1])] + ([d1] if self.lmax >= 1 else [])
        prev = d1
        for l in range(2, self.lmax + 1):
            c = self.cg[self.cg_starts[l]:self.cg_starts[l + 1]].view(2 * l + 1, 2 * l - 1, 3).to(rot.dtype)
            prev = torch.einsum("eakm,bkm->eab", torch.einsum("aij,eik,ejm->eakm", c, prev, d1), c)
            out.append(prev)
        return out


class Rotations(nn.Module):
    """Edge-frame rotation ``(E, R, (lmax+1)^2)`` into the truncated order-major layout and its
    inverse ``(E, (lmax+1)^2, R)`` (rows of degrees above ``mmax`` rescaled)."""

    def __init__(self, lmax: int, mmax: int):
        super().__init__()
        self.lmax, self.orders = int(lmax), _orders(lmax, mmax)
        self.rescaled = mmax < lmax
        scale = [s for l, s in enumerate(_rescale(lmax, mmax)) for _ in range(2 * self.orders[l] + 1)]
        order = m_primary_order(lmax, mmax)
        self.register_buffer("to_m", torch.tensor(order), persistent=False)
        self.register_buffer("from_m", torch.argsort(torch.tensor(order)), persistent=False)
        self.register_buffer("row_scales", torch.tensor([scale[i] for i in order], dtype=torch.float64), persistent=False)

    def matrices(self, wigner: List[Tensor]) -> Tuple[Tensor, Tensor]:
        full = (self.lmax + 1) ** 2
        rows = []
        for l, d in enumerate(wigner):
            mm = self.orders[l]
            rows.append(F.pad(d[:, l - mm:l + mm + 1], (l * l, full - (l + 1) ** 2)))
        rot = torch.cat(rows, 1).index_select(1, self.to_m)
        back = rot * self.row_scales.to(rot.dtype).unsqueeze(-1) if self.rescaled else rot
        return rot, back.transpose(1, 2)

    def gather_rotate(self, x: Tensor, src: Tensor, dst: Tensor, rot: Tensor) -> Tensor:
        return torch.bmm(rot, torch.cat([x.index_select(0, src), x.index_select(0, dst)], 2))

    def attend_rotate_back(self, msg: Tensor, attn: Tensor, rot_inv: Tensor, dst: Tensor, n: int) -> Tensor:
        e, r, hv = msg.shape
        h = attn.shape[1]
        weighted = (msg.view(e, r, h, hv // h) * attn[:, None, :, None]).reshape(e, r, hv)
        return scatter_sum(torch.bmm(rot_inv, weighted), dst, n)


class SO3Linear(nn.Module):
    """Per-degree channel mixing (a bias on the scalars)."""

    def __init__(self, in_features: int, out_features: int, lmax: int):
        super().__init__()
        self.in_features, self.out_features, self.lmax = in_features, out_features, int(lmax)
        bound = 1.0 / math.sqrt(in_features)
        self.weight = nn.Parameter(torch.empty(lmax + 1, out_features, in_features).uniform_(-bound, bound))
        self.bias = nn.Parameter(torch.zeros(out_features))

    def forward(self, x: Tensor) -> Tensor:
        out = [torch.matmul(x[:, l * l:(l + 1) ** 2], self.weight[l].t()) for l in range(self.lmax + 1)]
        out[0] = out[0] + self.bias
        return torch.cat(out, 1)


class SO2mConvolution(nn.Module):
    def __init__(self, in_features: int, out_features: int):
        super().__init__()
        self.fc = nn.Linear(in_features, 2 * out_features, bias=False)
        with torch.no_grad():
            self.fc.weight.mul_(1.0 / math.sqrt(2.0))


class SO2Convolution(nn.Module):
    """Linear maps per order on order-major edge features ``(E, R, C_in)``: a real map for ``m = 0``
    (with ``extra_m0`` extra scalar outputs, returned separately), a complex product of the
    ``(+m, -m)`` pair for ``m > 0``; inputs optionally weighted per channel by a radial MLP."""

    def __init__(self, in_channels: int, out_channels: int, lmax: int, mmax: int, radial: Optional[List[int]] = None,
                 extra_m0: int = 0, m_order_in: bool = False, m_order_out: bool = False):
        super().__init__()
        self.lmax, self.out_channels, self.extra_m0 = int(lmax), int(out_channels), int(extra_m0)
        self.m_order_in, self.m_order_out = m_order_in, m_order_out
        n0 = (lmax + 1) * in_channels
        self.fc_m0 = nn.Linear(n0, out_channels * (lmax + 1) + extra_m0)
        self.so2_m_conv = nn.ModuleList(SO2mConvolution((lmax - m + 1) * in_channels, (lmax - m + 1) * out_channels)
                                        for m in range(1, mmax + 1))
        self.w_sizes = [n0] + [(lmax - m + 1) * in_channels for m in range(1, mmax + 1)]
        self.x_sizes = [lmax + 1] + [2 * (lmax - m + 1) for m in range(1, mmax + 1)]
        self.rad_func = RadialMLP(list(radial) + [sum(self.w_sizes)]) if radial is not None else None
        order = m_primary_order(lmax, mmax)
        self.register_buffer("to_m", torch.tensor(order), persistent=False)
        self.register_buffer("from_m", torch.argsort(torch.tensor(order)), persistent=False)

    def forward(self, x: Tensor, x_edge: Tensor) -> Tuple[Tensor, Tensor]:
        e = x.shape[0]
        if not self.m_order_in:
            x = x.index_select(1, self.to_m)
        xs = torch.split(x, self.x_sizes, 1)
        ws = torch.split(self.rad_func(x_edge), self.w_sizes, 1) if self.rad_func is not None else None
        x0 = xs[0].reshape(e, -1)
        if ws is not None:
            x0 = x0 * ws[0]
        extra, y0 = torch.split(self.fc_m0(x0), [self.extra_m0, self.out_channels * (self.lmax + 1)], 1)
        outs = [y0.reshape(e, self.lmax + 1, self.out_channels)]
        for k, conv in enumerate(self.so2_m_conv):
            size = self.lmax - k
            xm = xs[k + 1].reshape(e, 2, -1)
            if ws is not None:
                xm = xm * ws[k + 1].unsqueeze(1)
            re, im = conv.fc(xm).chunk(2, dim=2)
            # (+m, -m) -> (re+ - im-, re- + im+)
            y = torch.stack([re[:, 0] - im[:, 1], re[:, 1] + im[:, 0]], 1)
            outs.append(y.reshape(e, 2 * size, self.out_channels))
        out = torch.cat(outs, 1)
        if not self.m_order_out:
            out = out.index_select(1, self.from_m)
        return out, extra


class GateActivation(nn.Module):
    """SiLU on the scalars, sigmoid gates (one per degree and channel) on the rest."""

    def __init__(self, lmax: int, mmax: int, channels: int):
        super().__init__()
        self.lmax, self.channels = int(lmax), int(channels)
        index = [l - 1 for l in range(1, lmax + 1) for _ in range(min(2 * l + 1, 2 * mmax + 1))]
        self.register_buffer("expand_index", torch.tensor(index, dtype=torch.long), persistent=False)

    def forward(self, gates: Tensor, x: Tensor) -> Tensor:
        g = torch.sigmoid(gates).view(gates.shape[0], self.lmax, self.channels).index_select(1, self.expand_index)
        return torch.cat([F.silu(x[:, :1]), x[:, 1:] * g], 1)


class SeparableS2Activation(nn.Module):
    def __init__(self, grid: S2Grid):
        super().__init__()
        self.grid = grid

    def forward(self, scalars: Tensor, x: Tensor) -> Tensor:
        out = self.grid(x)
        return torch.cat([F.silu(scalars).unsqueeze(1), out[:, 1:]], 1)


def _degree_list(lmax: int, start: int) -> List[int]:
    return [l for l in range(start, lmax + 1) for _ in range(2 * l + 1)]


class SeparableLayerNorm(nn.Module):
    """Layer norm of the scalars; the rest divided by the degree-balanced RMS over degrees >= 1."""

    def __init__(self, lmax: int, channels: int, eps: float = 1e-5):
        super().__init__()
        self.lmax, self.eps = int(lmax), float(eps)
        self.norm_l0 = nn.LayerNorm(channels, eps=eps)
        self.affine_weight = nn.Parameter(torch.ones(lmax, channels))
        w = [1.0 / ((2 * l + 1) * lmax) for l in _degree_list(lmax, 1)]
        self.register_buffer("balance_degree_weight", torch.tensor(w, dtype=torch.float64), persistent=False)
        self.register_buffer("expand_index", torch.tensor([l - 1 for l in _degree_list(lmax, 1)], dtype=torch.long),
                             persistent=False)

    def forward(self, x: Tensor) -> Tensor:
        out0 = self.norm_l0(x[:, :1])
        if self.lmax == 0:
            return out0
        rest = x[:, 1:]
        ms = torch.einsum("nic,i->nc", rest.pow(2), self.balance_degree_weight.to(x.dtype)).mean(1, keepdim=True)
        scale = (ms + self.eps).rsqrt().unsqueeze(1) * self.affine_weight.index_select(0, self.expand_index)
        return torch.cat([out0, rest * scale], 1)


class DegreeLayerNorm(nn.Module):
    """Each degree divided by its own RMS (the scalars centred first), per-degree affine weight."""

    def __init__(self, lmax: int, channels: int, eps: float = 1e-5):
        super().__init__()
        self.lmax, self.eps = int(lmax), float(eps)
        self.affine_weight = nn.Parameter(torch.ones(lmax + 1, channels))
        self.affine_bias = nn.Parameter(torch.zeros(channels))

    def forward(self, x: Tensor) -> Tensor:
        parts = []
        for l in range(self.lmax + 1):
            f = x[:, l * l:(l + 1) ** 2]
            if l == 0:
                f = f - f.mean(2, keepdim=True)
            ms = f.pow(2).mean(1, keepdim=True).mean(2, keepdim=True)
            f = f * ((ms + self.eps).rsqrt() * self.affine_weight[l].view(1, 1, -1))
            parts.append(f + self.affine_bias.view(1, 1, -1) if l == 0 else f)
        return torch.cat(parts, 1)


class RMSLayerNorm(nn.Module):
    """Scalars centred, then all degrees divided by one degree-balanced RMS."""

    def __init__(self, lmax: int, channels: int, eps: float = 1e-5):
        super().__init__()
        self.lmax, self.eps = int(lmax), float(eps)
        self.affine_weight = nn.Parameter(torch.ones(lmax + 1, channels))
        self.affine_bias = nn.Parameter(torch.zeros(channels))
        w = [1.0 / ((2 * l + 1) * (lmax + 1)) for l in _degree_list(lmax, 0)]
        self.register_buffer("balance_degree_weight", torch.tensor(w, dtype=torch.float64), persistent=False)
        self.register_buffer("expand_index", torch.tensor(_degree_list(lmax, 0), dtype=torch.long), persistent=False)

    def forward(self, x: Tensor) -> Tensor:
        x0 = x[:, :1]
        x = torch.cat([x0 - x0.mean(2, keepdim=True), x[:, 1:]], 1)
        ms = torch.einsum("nic,i->nc", x.pow(2), self.balance_degree_weight.to(x.dtype)).mean(1, keepdim=True)
        out = x * ((ms + self.eps).rsqrt().unsqueeze(1) * self.affine_weight.index_select(0, self.expand_index))
        return torch.cat([out[:, :1] + self.affine_bias, out[:, 1:]], 1)


def make_norm(kind: str, lmax: int, channels: int) -> nn.Module:
    if kind == "layer_norm_sh":
        return SeparableLayerNorm(lmax, channels)
    if kind == "layer_norm":
        return DegreeLayerNorm(lmax, channels)
    if kind == "rms_norm_sh":
        return RMSLayerNorm(lmax, channels)
    raise ValueError(f"norm_type must be one of {NORMS}, got {kind!r}")


class EdgeScalars(nn.Module):
    """Radial features, optionally with source and target element embeddings appended."""

    def __init__(self, n_elements: int, channels: int, use_elements: bool):
        super().__init__()
        self.source_embedding = self.target_embedding = None
        if use_elements:
            self.source_embedding = nn.Embedding(n_elements, channels)
            self.target_embedding = nn.Embedding(n_elements, channels)
            nn.init.uniform_(self.source_embedding.weight, -0.001, 0.001)
            nn.init.uniform_(self.target_embedding.weight, -0.001, 0.001)

    def forward(self, rbf: Tensor, z: Tensor, src: Tensor, dst: Tensor) -> Tensor:
        if self.source_embedding is None:
            return rbf
        return torch.cat([rbf, self.source_embedding(z[src]), self.target_embedding(z[dst])], 1)


class SO2GraphAttention(nn.Module):
    """Rotate both ends into the edge frame, SO(2) convolution (radial weights, attention scalars
    on the side), activation, second SO(2) convolution to the value heads, softmax over each
    receiver's edges (envelope-weighted when smooth), rotate back, sum, per-degree projection."""

    def __init__(self, channels: int, hidden_channels: int, num_heads: int, alpha_channels: int, value_channels: int,
                 out_channels: int, lmax: int, mmax: int, radial: List[int], n_elements: int,
                 use_atom_edge_embedding: bool, use_m_share_rad: bool, activation: str, use_attn_renorm: bool,
                 resolution: Optional[int], alpha_drop: float = 0.0):
        super().__init__()
        if activation not in ACTIVATIONS:
            raise ValueError(f"activation must be one of {ACTIVATIONS}, got {activation!r}")
        self.num_heads, self.alpha_channels, self.lmax = int(num_heads), int(alpha_channels), int(lmax)
        radial = list(radial)
        self.edge_scalars = EdgeScalars(n_elements, radial[-1], use_atom_edge_embedding)
        if use_atom_edge_embedding:
            radial[0] += 2 * radial[-1]
        extra = num_heads * alpha_channels + {"gate": lmax * hidden_channels, "sep_s2": hidden_channels}.get(activation, 0)
        self.rad_func = None
        if use_m_share_rad:
            self.rad_func = RadialMLP(radial + [2 * channels * (lmax + 1)])
            degree = [l for l, mm in enumerate(_orders(lmax, mmax)) for _ in range(2 * mm + 1)]
            self.register_buffer("expand_index", torch.tensor([degree[i] for i in m_primary_order(lmax, mmax)]),
                                 persistent=False)
        self.rotations = Rotations(lmax, mmax)
        self.so2_conv_1 = SO2Convolution(2 * channels, hidden_channels, lmax, mmax, None if use_m_share_rad else radial,
                                         extra, m_order_in=True)
        self.alpha_norm = nn.LayerNorm(alpha_channels) if use_attn_renorm else nn.Identity()
        self.alpha_act = SmoothLeakyReLU(0.2)
        bound = 1.0 / math.sqrt(alpha_channels)
        self.alpha_dot = nn.Parameter(torch.empty(num_heads, alpha_channels).uniform_(-bound, bound))
        self.alpha_dropout = nn.Dropout(alpha_drop) if alpha_drop > 0 else nn.Identity()
        self.gate_act = self.s2_act = self.grid = None
        if activation == "gate":
            self.gate_act = GateActivation(lmax, mmax, hidden_channels)
        elif activation == "sep_s2":
            self.s2_act = SeparableS2Activation(S2Grid(lmax, mmax, resolution))
        else:
            self.grid = S2Grid(lmax, mmax, resolution)
        self.so2_conv_2 = SO2Convolution(hidden_channels, num_heads * value_channels, lmax, mmax, m_order_out=True)
        self.proj = SO3Linear(num_heads * value_channels, out_channels, lmax)

    def forward(self, x: Tensor, z: Tensor, edge_rbf: Tensor, src: Tensor, dst: Tensor, rot: Tensor, rot_inv: Tensor,
                envelope: Optional[Tensor]) -> Tensor:
        n, e = x.shape[0], src.shape[0]
        x_edge = self.edge_scalars(edge_rbf, z, src, dst)
        msg = self.rotations.gather_rotate(x, src, dst, rot)
        if self.rad_func is not None:
            msg = msg * self.rad_func(x_edge).view(e, self.lmax + 1, -1).index_select(1, self.expand_index)
        msg, extra = self.so2_conv_1(msg, x_edge)
        n_alpha = self.num_heads * self.alpha_channels
        alpha, side = extra[:, :n_alpha], extra[:, n_alpha:]
        if self.gate_act is not None:
            msg = self.gate_act(side, msg)
        elif self.s2_act is not None:
            msg = self.s2_act(side, msg)
        else:
            msg = self.grid(msg)
        msg, _ = self.so2_conv_2(msg, x_edge)
        alpha = self.alpha_act(self.alpha_norm(alpha.view(e, self.num_heads, self.alpha_channels)))
        attn = self.alpha_dropout(segment_softmax(torch.einsum("ehk,hk->eh", alpha, self.alpha_dot), dst, n, envelope))
        return self.proj(self.rotations.attend_rotate_back(msg, attn, rot_inv, dst, n))


class FeedForwardNetwork(nn.Module):
    """Per-degree linear, a nonlinearity (an MLP on the S2 grid, a gate, the separable or plain
    grid SiLU), per-degree linear."""

    def __init__(self, channels: int, hidden_channels: int, out_channels: int, lmax: int, activation: str,
                 use_grid_mlp: bool, resolution: Optional[int]):
        super().__init__()
        if activation not in ACTIVATIONS:
            raise ValueError(f"activation must be one of {ACTIVATIONS}, got {activation!r}")
        self.so3_linear_1 = SO3Linear(channels, hidden_channels, lmax)
        self.grid = self.scalar_mlp = self.grid_mlp = self.gating_linear = self.gate_act = self.s2_act = None
        if use_grid_mlp:
            self.grid = S2Grid(lmax, lmax, resolution)
            if activation == "sep_s2":
                self.scalar_mlp = nn.Sequential(nn.Linear(channels, hidden_channels), nn.SiLU())
            self.grid_mlp = nn.Sequential(nn.Linear(hidden_channels, hidden_channels, bias=False), nn.SiLU(),
                                          nn.Linear(hidden_channels, hidden_channels, bias=False), nn.SiLU(),
                                          nn.Linear(hidden_channels, hidden_channels, bias=False))
        elif activation == "gate":
            self.gating_linear = nn.Linear(channels, lmax * hidden_channels)
            self.gate_act = GateActivation(lmax, lmax, hidden_channels)
        elif activation == "sep_s2":
            self.gating_linear = nn.Linear(channels, hidden_channels)
            self.s2_act = SeparableS2Activation(S2Grid(lmax, lmax, resolution))
        else:
            self.grid = S2Grid(lmax, lmax, resolution)
        self.so3_linear_2 = SO3Linear(hidden_channels, out_channels, lmax)

    def forward(self, x: Tensor) -> Tensor:
        x0 = x[:, 0]
        h = self.so3_linear_1(x)
        if self.grid_mlp is not None:
            h = self.grid.from_grid(self.grid_mlp(self.grid.to_grid(h)))
            if self.scalar_mlp is not None:
                h = torch.cat([self.scalar_mlp(x0).unsqueeze(1), h[:, 1:]], 1)
        elif self.gate_act is not None:
            h = self.gate_act(self.gating_linear(x0), h)
        elif self.s2_act is not None:
            h = self.s2_act(self.gating_linear(x0), h)
        else:
            h = self.grid(h)
        return self.so3_linear_2(h)


class EquivariantDropout(nn.Module):
    """One dropout mask per node and channel, shared by all coefficients."""

    def __init__(self, p: float):
        super().__init__()
        self.p = float(p)

    def forward(self, x: Tensor) -> Tensor:
        if not self.training or self.p == 0.0:
            return x
        return x * F.dropout(x.new_ones((x.shape[0], 1, x.shape[2])), self.p, True)


class TransformerBlockV2(nn.Module):
    def __init__(self, channels: int, attn_hidden_channels: int, num_heads: int, attn_alpha_channels: int,
                 attn_value_channels: int, ffn_hidden_channels: int, lmax: int, mmax: int, radial: List[int],
                 n_elements: int, use_atom_edge_embedding: bool, use_m_share_rad: bool, activation: str,
                 use_attn_renorm: bool, use_grid_mlp: bool, norm_type: str, resolution: Optional[int],
                 alpha_drop: float, drop_path_rate: float, proj_drop: float):
        super().__init__()
        self.norm_1 = make_norm(norm_type, lmax, channels)
        self.ga = SO2GraphAttention(channels, attn_hidden_channels, num_heads, attn_alpha_channels, attn_value_channels,
                                    channels, lmax, mmax, radial, n_elements, use_atom_edge_embedding, use_m_share_rad,
                                    activation, use_attn_renorm, resolution, alpha_drop)
        self.drop_path = GraphDropPath(drop_path_rate)
        self.proj_drop = EquivariantDropout(proj_drop)
        self.norm_2 = make_norm(norm_type, lmax, channels)
        self.ffn = FeedForwardNetwork(channels, ffn_hidden_channels, channels, lmax, activation, use_grid_mlp,
                                      resolution)

    def forward(self, x, z, edge_rbf, src, dst, rot, rot_inv, envelope, batch, num_graphs: int):
        h = self.ga(self.norm_1(x), z, edge_rbf, src, dst, rot, rot_inv, envelope)
        x = x + self.proj_drop(self.drop_path(h, batch, num_graphs))
        return x + self.proj_drop(self.drop_path(self.ffn(self.norm_2(x)), batch, num_graphs))


class EdgeDegreeEmbedding(nn.Module):
    """Initial non-scalar features: each edge's radial coefficients placed on the ``m = 0`` column
    of its frame's Wigner matrices (the frame rotated back), summed per receiver."""

    def __init__(self, channels: int, lmax: int, mmax: int, radial: List[int], n_elements: int,
                 use_atom_edge_embedding: bool, avg_degree: float):
        super().__init__()
        self.lmax, self.channels = int(lmax), int(channels)
        radial = list(radial)
        self.edge_scalars = EdgeScalars(n_elements, radial[-1], use_atom_edge_embedding)
        if use_atom_edge_embedding:
            radial[0] += 2 * radial[-1]
        self.rad_func = RadialMLP(radial + [(lmax + 1) * channels])
        self.scales = _rescale(lmax, mmax)
        self.avg_degree = float(avg_degree)

    def forward(self, z, edge_rbf, src, dst, wigner: List[Tensor], n: int, envelope: Optional[Tensor]) -> Tensor:
        coef = self.rad_func(self.edge_scalars(edge_rbf, z, src, dst)).view(src.shape[0], self.lmax + 1, self.channels)
        if envelope is not None:
            coef = coef * envelope[:, None, None]
        parts = [d[:, l].unsqueeze(-1) * (coef[:, l:l + 1] * self.scales[l]) for l, d in enumerate(wigner)]
        return scatter_sum(torch.cat(parts, 1), dst, n) / self.avg_degree


def _init_weights(module: nn.Module, weight_init: str) -> None:
    radial = set()
    for m in module.modules():
        if isinstance(m, RadialMLP):
            for lin in m.modules():
                if isinstance(lin, nn.Linear):
                    radial.add(id(lin))
                    nn.init.uniform_(lin.weight, -1.0 / math.sqrt(lin.in_features), 1.0 / math.sqrt(lin.in_features))
                    if lin.bias is not None:
                        nn.init.zeros_(lin.bias)
    for m in module.modules():
        if isinstance(m, (nn.Linear, SO3Linear)) and id(m) not in radial:
            if m.bias is not None:
                nn.init.zeros_(m.bias)
            if weight_init == "normal":
                nn.init.normal_(m.weight, 0.0, 1.0 / math.sqrt(m.in_features))
        elif isinstance(m, nn.LayerNorm):
            nn.init.ones_(m.weight)
            nn.init.zeros_(m.bias)


@register_model("equiformer_v2")
class EquiformerV2(TransformerPotential):
    """EquiformerV2 energy model (``direct_forces``: an extra attention block predicts forces from
    its ``l = 1`` output; the energy is then not their potential)."""
    head_modules = ("energy_block", "energy_scale", "energy_shift", "atom_ref")

    def __init__(self, n_features: int = 96, n_interactions: int = 6, cutoff: float = 5.0, n_rbf: int = 128,
                 l_max: int = 4, m_max: int = 4, num_heads: int = 4, attn_hidden_channels: int = 48,
                 attn_alpha_channels: int = 64, attn_value_channels: int = 24, ffn_hidden_channels: int = 96,
                 edge_channels: int = 64, norm_type: str = "layer_norm_sh", activation: str = "sep_s2",
                 use_grid_mlp: bool = True, use_attn_renorm: bool = True, use_atom_edge_embedding: bool = True,
                 share_atom_edge_embedding: bool = False, use_m_share_rad: bool = False,
                 grid_resolution: Optional[int] = 18, alpha_drop: float = 0.0, drop_path_rate: float = 0.0,
                 proj_drop: float = 0.0, avg_degree: float = AVG_DEGREE, avg_num_nodes: float = AVG_NUM_NODES,
                 direct_forces: bool = False, smooth_cutoff: bool = False, weight_init: str = "normal",
                 n_elements: int = 100, energy_shift: float = 0.0, energy_scale: float = 1.0, species=None,
                 atomic_energies=None):
        super().__init__()
        if not 0 <= m_max <= l_max:
            raise ValueError(f"need 0 <= m_max <= l_max, got m_max={m_max}, l_max={l_max}")
        if norm_type not in NORMS:
            raise ValueError(f"norm_type must be one of {NORMS}, got {norm_type!r}")
        if weight_init not in ("normal", "uniform"):
            raise ValueError(f"weight_init must be 'normal' or 'uniform', got {weight_init!r}")
        self.cutoff = float(cutoff)
        if species is not None:
            self.species = [int(z) for z in species]
        self.n_features = self.node_feature_dim = int(n_features)
        self.n_interactions = int(n_interactions)
        self.lmax, self.mmax = int(l_max), int(m_max)
        self.avg_num_nodes, self.smooth, self.direct_forces = float(avg_num_nodes), bool(smooth_cutoff), bool(direct_forces)
        spacing = cutoff / (n_rbf - 1) if n_rbf > 1 else 1.0
        self.distance_expansion = GaussianRBF(n_rbf, cutoff, gamma=0.5 / (2.0 * spacing) ** 2)
        self.envelope = PolynomialCutoff(cutoff, p=6)
        radial = [n_rbf, edge_channels, edge_channels]
        self.shared_edge_scalars = EdgeScalars(n_elements, edge_channels, share_atom_edge_embedding)
        per_block = use_atom_edge_embedding and not share_atom_edge_embedding
        if share_atom_edge_embedding:
            radial[0] += 2 * edge_channels
        self.sphere_embedding = nn.Embedding(n_elements, n_features)
        self.frames = EdgeFrames(l_max)
        self.rotations = Rotations(l_max, m_max)
        self.edge_degree_embedding = EdgeDegreeEmbedding(n_features, l_max, m_max, radial, n_elements, per_block,
                                                         avg_degree)
        self.blocks = nn.ModuleList(TransformerBlockV2(
            n_features, attn_hidden_channels, num_heads, attn_alpha_channels, attn_value_channels, ffn_hidden_channels,
            l_max, m_max, radial, n_elements, per_block, use_m_share_rad, activation, use_attn_renorm, use_grid_mlp,
            norm_type, grid_resolution, alpha_drop, drop_path_rate, proj_drop) for _ in range(n_interactions))
        self.norm = make_norm(norm_type, l_max, n_features)
        self.energy_block = FeedForwardNetwork(n_features, ffn_hidden_channels, 1, l_max, activation, use_grid_mlp,
                                               grid_resolution)
        self.force_block = None
        if self.direct_forces:
            self.force_block = SO2GraphAttention(
                n_features, attn_hidden_channels, num_heads, attn_alpha_channels, attn_value_channels, 1, l_max, m_max,
                radial, n_elements, per_block, use_m_share_rad, activation, use_attn_renorm, grid_resolution, 0.0)
        _init_weights(self, weight_init)
        self._init_energy_terms(n_elements, energy_scale, energy_shift, species, atomic_energies)

    def receptive_field(self) -> float:
        return self.n_interactions * self.cutoff

    def _evaluate(self, z: Tensor, edge_index: Tensor, edge_vec: Tensor, batch: Tensor, num_graphs: int):
        n = z.shape[0]
        src, dst = edge_index[0], edge_index[1]
        vec = -edge_vec
        r = torch.linalg.norm(vec, dim=-1)
        wigner = self.frames(vec)
        rot, rot_inv = self.rotations.matrices(wigner)
        edge_rbf = self.shared_edge_scalars(self.distance_expansion(r), z, src, dst)
        envelope = self.envelope(r) if self.smooth else None
        x0 = self.sphere_embedding(z).unsqueeze(1)
        x = torch.cat([x0, x0.new_zeros((n, (self.lmax + 1) ** 2 - 1, self.n_features))], 1)
        x = x + self.edge_degree_embedding(z, edge_rbf, src, dst, wigner, n, envelope)
        for block in self.blocks:
            x = block(x, z, edge_rbf, src, dst, rot, rot_inv, envelope, batch, num_graphs)
        x = self.norm(x)
        y = self.energy_block(x)[:, 0, 0] / self.avg_num_nodes
        forces = None
        if self.force_block is not None:
            out = self.force_block(x, z, edge_rbf, src, dst, rot, rot_inv, envelope)
            forces = out[:, 1:4, 0] @ self.frames.basis.to(out.dtype)
        return x, y, forces

    def _energy(self, y: Tensor, z: Tensor) -> Tensor:
        return self.energy_scale * y + self.energy_shift + self.atom_ref(z).squeeze(-1)

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        if self.direct_forces:
            raise RuntimeError("an EquiformerV2 with direct_forces has no energy-only core "
                               "(its forces are not the gradient of the energy)")
        x, y, _ = self._evaluate(atomic_numbers, edge_index, edge_vec, torch.zeros_like(atomic_numbers), 1)
        return x[:, 0], self._energy(y, atomic_numbers)

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        x, y, forces = self._evaluate(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.batch,
                                      data.num_graphs)
        node = self._energy(y, data.atomic_numbers)
        out = {"node_energy": node, "energy": self.aggregate_energy(node, data), "node_features": x[:, 0]}
        if forces is not None:
            out["forces"] = forces.to(data.pos.dtype)
        return out

    @classmethod
    def from_config(cls, cfg) -> "EquiformerV2":
        e = dict(cfg.extra or {})
        kw = {}
        for key in ("l_max", "m_max"):
            if key in e:
                v = e[key]
                if isinstance(v, (list, tuple)):
                    if len(v) != 1:
                        raise ValueError(f"{key}: one resolution is supported, got {v}")
                    v = v[0]
                kw[key] = int(v)
        for key, kind in (("num_heads", int), ("attn_hidden_channels", int), ("attn_alpha_channels", int),
                          ("attn_value_channels", int), ("ffn_hidden_channels", int), ("edge_channels", int),
                          ("norm_type", str), ("activation", str), ("use_grid_mlp", bool), ("use_attn_renorm", bool),
                          ("use_atom_edge_embedding", bool), ("share_atom_edge_embedding", bool),
                          ("use_m_share_rad", bool), ("alpha_drop", float), ("drop_path_rate", float),
                          ("proj_drop", float), ("avg_degree", float), ("avg_num_nodes", float), ("direct_forces", bool),
                          ("smooth_cutoff", bool), ("weight_init", str), ("n_elements", int), ("energy_shift", float),
                          ("energy_scale", float)):
            if e.get(key) is not None:
                kw[key] = kind(e[key])
        if "grid_resolution" in e:
            kw["grid_resolution"] = None if e["grid_resolution"] is None else int(e["grid_resolution"])
        for key in ("species", "atomic_energies"):
            if e.get(key) is not None:
                kw[key] = e[key]
        return cls(n_features=cfg.n_features, n_interactions=cfg.n_interactions, cutoff=cfg.cutoff, n_rbf=cfg.n_rbf,
                   **kw)
