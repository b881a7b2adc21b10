"""Equiformer (Liao & Smidt, ICLR 2023): an equivariant graph-attention transformer on irreps
features. Pre-norm blocks: equivariant layer norm, graph attention, residual; layer norm,
gated feed-forward, residual. The attention mixes the edge's two ends (``Linear_src(x_j) +
Linear_dst(x_i)``), takes a depth-wise (``uvu``) tensor product with the edge's spherical
harmonics weighted by a radial MLP, and forms MLP attention logits from its scalars (non-linear
messages gate the result and take a second depth-wise product) or dot-product attention; the
embedding adds a degree embedding; the energy is a gated readout of the final scalars divided by
``sqrt(avg_num_nodes)``.

Layouts, normalisations, presets and parameter names follow the reference
(``src/xnn/trfnn/models/equiformer.py``) so state dicts transplant; SH on ``r_j - r_i``; the
``smooth_cutoff`` option weights the attention by a polynomial envelope with a null key.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn import PolynomialCutoff
from ..nn.radial import BesselRBF, ExpNormalSmearing
from ..o3 import Irrep, Irreps, SphericalHarmonics, TensorProduct, normalize2mom
from ..ops.scatter import scatter_sum, segment_softmax
from .et import TransformerPotential
from .registry import register_model

AVG_NUM_NODES = 18.03065905448718
AVG_DEGREE = 15.57930850982666
_SQRT_2PI = (2 * 3.14159) ** 0.5
PRESETS = {
    (1, False): ("256x0e+128x1e", "32x0e+16x1e", 8, "768x0e+384x1e"),
    (2, False): ("128x0e+64x1e+32x2e", "32x0e+16x1e+8x2e", 4, "384x0e+192x1e+96x2e"),
    (3, False): ("128x0e+64x1e+64x2e+32x3e", "32x0e+16x1e+16x2e+8x3e", 4, "384x0e+192x1e+192x2e+96x3e"),
    (1, True): ("256x0e+64x0o+64x1e+64x1o", "32x0e+8x0o+8x1e+8x1o", 8, "768x0e+192x0o+192x1e+192x1o"),
    (2, True): ("128x0e+32x0o+32x1e+32x1o+16x2e+16x2o", "32x0e+8x0o+8x1e+8x1o+4x2e+4x2o", 4,
                "384x0e+96x0o+96x1e+96x1o+48x2e+48x2o"),
    (3, True): ("128x0e+64x0o+32x1e+32x1o+32x2e+32x2o+16x3e+16x3o", "32x0e+16x0o+8x1e+8x1o+8x2e+8x2o+4x3e+4x3o", 4,
                "384x0e+192x0o+96x1e+96x1o+96x2e+96x2o+48x3e+48x3o"),
}


def paper_irreps(l_max: int = 2, e3: bool = False, n_features: Optional[int] = None) -> Dict[str, object]:
    """The paper's irreps (node, head, heads, FFN middle), rescaled to ``n_features`` scalars."""
    if (l_max, e3) not in PRESETS:
        raise ValueError(f"no preset for l_max={l_max}, e3={e3}")
    emb, head, heads, mid = PRESETS[(l_max, e3)]
    if n_features is not None:
        base = Irreps(emb)[0].mul

        def scale(irreps):
            out = Irreps([(mul * n_features // base, ir) for mul, ir in Irreps(irreps)])
            if any(mul == 0 for mul, _ in out):
                raise ValueError(f"n_features={n_features} leaves {irreps} with an empty irrep")
            return str(out)
        emb, head, mid = scale(emb), scale(head), scale(mid)
    return {"irreps_node_embedding": emb, "irreps_head": head, "num_heads": heads, "irreps_mlp_mid": mid}


def moment_scale(fn) -> float:
    """The factor normalising the second moment of ``fn`` on a standard normal."""
    norm = normalize2mom(fn)
    return 1.0 if getattr(norm, "_is_id", False) else float(norm.cst)


def sort_even_first(irreps: Irreps) -> Tuple[Irreps, List[int]]:
    keys = sorted((ir.l, -ir.p, i, mul) for i, (mul, ir) in enumerate(irreps))
    new_of_old = [0] * len(keys)
    for new, (_, _, old, _) in enumerate(keys):
        new_of_old[old] = new
    return Irreps([(mul, (l, -negp)) for l, negp, _, mul in keys]), new_of_old


def sort_irreps(irreps: Irreps, even_first: bool) -> Irreps:
    return sort_even_first(irreps)[0].simplify() if even_first else irreps.sort()[0].simplify()


def irreps_to_gate(irreps: Irreps):
    scalars = Irreps([(m, ir) for m, ir in irreps if ir.l == 0 and ir.p == 1]).simplify()
    gated = Irreps([(m, ir) for m, ir in irreps if not (ir.l == 0 and ir.p == 1)]).simplify()
    return scalars, Irreps([(m, "0e") for m, _ in gated]).simplify(), gated


def depthwise_tensor_product(irreps_in, irreps_sh, irreps_target, internal_weights: bool) -> TensorProduct:
    """One weight per channel and path (``uvu``) to the target degrees and even scalars, outputs
    sorted by degree (even first); shared weights scaled by ``fan_in^-1/2``."""
    irreps_in, irreps_sh, target = Irreps(irreps_in), Irreps(irreps_sh), Irreps(irreps_target)
    outs, instr = [], []
    for i, (mul, ir_in) in enumerate(irreps_in):
        for j, (_, ir_sh) in enumerate(irreps_sh):
            for ir_out in ir_in * ir_sh:
                if ir_out in target or ir_out == Irrep(0, 1):
                    instr.append((i, j, len(outs), "uvu", True))
                    outs.append((mul, ir_out))
    irreps_out, new_of_old = sort_even_first(Irreps(outs))
    instr = [(i, j, new_of_old[k], m, t) for i, j, k, m, t in instr]
    tp = TensorProduct(irreps_in, irreps_sh, irreps_out, instr, internal_weights=internal_weights,
                       shared_weights=internal_weights, irrep_normalization="component", path_normalization="none")
    if internal_weights:
        with torch.no_grad():
            for w, ins in zip(tp.weight_views(), tp.instructions):
                w.mul_(sum(irreps_sh[o.i_in2].mul for o in tp.instructions if o.i_out == ins.i_out) ** -0.5)
    return tp


class IrrepsLinear(nn.Module):
    """One weight matrix per pair of equal irreps (flat, input-major), ``fan_in^-1/2`` at init, a bias
    on the even scalars."""

    def __init__(self, irreps_in, irreps_out, bias: bool = True):
        super().__init__()
        self.irreps_in, self.irreps_out = Irreps(irreps_in), Irreps(irreps_out)
        starts = [0]
        for mul, ir in self.irreps_in:
            starts.append(starts[-1] + mul * ir.dim)
        paths, w = [], 0
        for i, (mi, iri) in enumerate(self.irreps_in):
            for o, (mo, iro) in enumerate(self.irreps_out):
                if iri == iro and mi > 0 and mo > 0:
                    paths.append((o, starts[i], mi, w))
                    w += mi * mo
        paths.sort(key=lambda p: p[0])
        self.paths = paths
        self.out = [(mul, ir.dim) for mul, ir in self.irreps_out]
        self.weight = nn.Parameter(torch.randn(w))
        with torch.no_grad():
            for o, (mo, _) in enumerate(self.out):
                mine = [p for p in paths if p[0] == o]
                fan_in = sum(p[2] for p in mine)
                for _, _, mi, ws in mine:
                    self.weight.narrow(0, ws, mi * mo).mul_(fan_in ** -0.5)
        scalars = [o for o, (_, ir) in enumerate(self.irreps_out) if ir == Irrep(0, 1)]
        if len(scalars) > 1:
            raise ValueError(f"expected one even-scalar output entry, got {self.irreps_out}")
        self.bias_entry = scalars[0] if bias and scalars else -1
        self.bias = nn.Parameter(torch.zeros(self.out[self.bias_entry][0])) if self.bias_entry >= 0 else None

    def forward(self, x: Tensor) -> Tensor:
        n, parts = x.shape[0], []
        for o, (mo, d) in enumerate(self.out):
            y = x.new_zeros((n, mo, d))
            for po, start, mi, ws in self.paths:
                if po == o:
                    y = y + torch.einsum("nud,uw->nwd", x.narrow(1, start, mi * d).reshape(n, mi, d),
                                         self.weight.narrow(0, ws, mi * mo).view(mi, mo))
            y = y.reshape(n, mo * d)
            if o == self.bias_entry:
                y = y + self.bias
            parts.append(y)
        return torch.cat(parts, 1)


class EquivariantLayerNorm(nn.Module):
    """Per irreps entry: even scalars centred over channels; every entry divided by the RMS of its
    component-normalised norms and scaled per channel; a bias on the even scalars."""

    def __init__(self, irreps, eps: float = 1e-5):
        super().__init__()
        self.irreps, self.eps = Irreps(irreps), float(eps)
        self.entries, x, w, b = [], 0, 0, 0
        for mul, ir in self.irreps:
            sc = ir.l == 0 and ir.p == 1
            self.entries.append((x, mul, ir.dim, sc, w, b))
            x, w, b = x + mul * ir.dim, w + mul, b + (mul if sc else 0)
        self.affine_weight = nn.Parameter(torch.ones(w))
        self.affine_bias = nn.Parameter(torch.zeros(b))

    def forward(self, x: Tensor) -> Tensor:
        out = []
        for start, mul, d, sc, ws, bs in self.entries:
            f = x.narrow(1, start, mul * d).reshape(-1, mul, d)
            if sc:
                f = f - f.mean(1, keepdim=True)
            norm = (f.pow(2).mean(-1).mean(1, keepdim=True) + self.eps).pow(-0.5) * self.affine_weight[ws:ws + mul][None]
            f = f * norm.reshape(-1, mul, 1)
            if sc:
                f = f + self.affine_bias[bs:bs + mul].reshape(mul, 1)
            out.append(f.reshape(-1, mul * d))
        return torch.cat(out, -1)


class Gate(nn.Module):
    """Normalised SiLU on even scalars, normalised sigmoid gates on the other irreps."""

    def __init__(self, irreps_out):
        super().__init__()
        scalars, gates, gated = irreps_to_gate(Irreps(irreps_out))
        self.has_gates = gated.num_irreps > 0
        self.irreps_out = (scalars + gated).simplify() if self.has_gates else Irreps(irreps_out)
        self.irreps_in = (scalars + gates + gated).simplify() if self.has_gates else self.irreps_out
        self.n_scalars = scalars.dim if self.has_gates else self.irreps_out.dim
        self.n_gates = gates.dim
        self.gated = [(mul, ir.dim) for mul, ir in gated]
        self.silu_scale, self.sigmoid_scale = moment_scale(F.silu), moment_scale(torch.sigmoid)

    def forward(self, x: Tensor) -> Tensor:
        if not self.has_gates:
            return F.silu(x) * self.silu_scale
        parts = [F.silu(x[:, :self.n_scalars]) * self.silu_scale]
        gates = torch.sigmoid(x[:, self.n_scalars:self.n_scalars + self.n_gates]) * self.sigmoid_scale
        at, g = self.n_scalars + self.n_gates, 0
        for mul, d in self.gated:
            parts.append((x[:, at:at + mul * d].reshape(-1, mul, d) * gates[:, g:g + mul, None]).reshape(-1, mul * d))
            at, g = at + mul * d, g + mul
        return torch.cat(parts, 1)


class ChannelDropout(nn.Module):
    def __init__(self, irreps, p: float):
        super().__init__()
        self.p, self.fields = float(p), [(mul, ir.dim) for mul, ir in Irreps(irreps)]

    def forward(self, x: Tensor) -> Tensor:
        if not self.training or self.p == 0.0:
            return x
        n = x.shape[0]
        mask = F.dropout(x.new_ones((n, sum(m for m, _ in self.fields))), self.p, True)
        parts, at, c = [], 0, 0
        for mul, d in self.fields:
            parts.append((x[:, at:at + mul * d].reshape(n, mul, d) * mask[:, c:c + mul, None]).reshape(n, mul * d))
            at, c = at + mul * d, c + mul
        return torch.cat(parts, 1)


class Heads(nn.Module):
    """Split ``(n, h * width)`` irreps features into ``(n, h, width)`` per-head blocks and back."""

    def __init__(self, irreps_head, num_heads: int):
        super().__init__()
        self.widths, self.num_heads = [mul * ir.dim for mul, ir in Irreps(irreps_head)], int(num_heads)

    def split(self, x: Tensor) -> Tensor:
        n, h, parts, at = x.shape[0], self.num_heads, [], 0
        for w in self.widths:
            parts.append(x[:, at:at + w * h].reshape(n, h, w))
            at += w * h
        return torch.cat(parts, 2)

    def merge(self, x: Tensor) -> Tensor:
        n, h, parts, at = x.shape[0], self.num_heads, [], 0
        for w in self.widths:
            parts.append(x[:, :, at:at + w].reshape(n, h * w))
            at += w
        return torch.cat(parts, 1)


class RadialMLP(nn.Module):
    """Linear, LayerNorm, SiLU between layers."""

    def __init__(self, channels: List[int]):
        super().__init__()
        layers = []
        for k in range(1, len(channels)):
            layers.append(nn.Linear(channels[k - 1], channels[k]))
            if k < len(channels) - 1:
                layers += [nn.LayerNorm(channels[k]), nn.SiLU()]
        self.net = nn.Sequential(*layers)

    def forward(self, x: Tensor) -> Tensor:
        return self.net(x)


class SmoothLeakyReLU(nn.Module):
    def __init__(self, negative_slope: float = 0.2):
        super().__init__()
        self.alpha = float(negative_slope)

    def forward(self, x: Tensor) -> Tensor:
        return 0.5 * (1.0 + self.alpha) * x + 0.5 * (1.0 - self.alpha) * x * (2.0 * torch.sigmoid(x) - 1.0)


class GraphDropPath(nn.Module):
    def __init__(self, drop_prob: float):
        super().__init__()
        self.drop_prob = float(drop_prob)

    def forward(self, x: Tensor, batch: Tensor, num_graphs: int) -> Tensor:
        if self.drop_prob == 0.0 or not self.training:
            return x
        keep = 1.0 - self.drop_prob
        mask = torch.floor(keep + torch.rand(num_graphs, dtype=x.dtype, device=x.device)) / keep
        return x * mask[batch].reshape([x.shape[0]] + [1] * (x.dim() - 1))


class GaussianBasis(nn.Module):
    def __init__(self, n_rbf: int, cutoff: float):
        super().__init__()
        self.n_rbf, self.cutoff = n_rbf, float(cutoff)
        self.mean = nn.Parameter(torch.empty(1, n_rbf).uniform_(0.0, 1.0))
        self.std = nn.Parameter(torch.empty(1, n_rbf).uniform_(1.0 / n_rbf, 1.0))
        self.weight = nn.Parameter(torch.ones(1, 1))
        self.bias = nn.Parameter(torch.zeros(1, 1))

    def forward(self, r: Tensor) -> Tensor:
        x = (self.weight * (r / self.cutoff).unsqueeze(-1) + self.bias).expand(-1, self.n_rbf)
        std = self.std.abs() + 1e-5
        return torch.exp(-0.5 * ((x - self.mean) / std) ** 2) / (_SQRT_2PI * std)


class BesselBasis(nn.Module):
    def __init__(self, n_rbf: int, cutoff: float):
        super().__init__()
        self.rbf = BesselRBF(n_rbf, cutoff, trainable=True)
        self.envelope = PolynomialCutoff(cutoff, p=5)

    def forward(self, r: Tensor) -> Tensor:
        return self.envelope(r).unsqueeze(-1) * self.rbf(r)


def make_radial_basis(name: str, n_rbf: int, cutoff: float) -> nn.Module:
    if name == "expnorm":
        return ExpNormalSmearing(n_rbf, cutoff, trainable=False)
    if name == "gaussian":
        return GaussianBasis(n_rbf, cutoff)
    if name == "bessel":
        return BesselBasis(n_rbf, cutoff)
    raise ValueError(f"radial_basis must be 'expnorm', 'gaussian' or 'bessel', got {name!r}")


class SeparableTP(nn.Module):
    """Depth-wise tensor product (radial-weighted per edge, or shared weights) then a linear map."""

    def __init__(self, irreps_in, irreps_sh, irreps_target, irreps_lin_out, radial: Optional[List[int]]):
        super().__init__()
        self.dtp = depthwise_tensor_product(irreps_in, irreps_sh, irreps_target, internal_weights=radial is None)
        self.rad = RadialMLP(radial + [self.dtp.weight_numel]) if radial is not None else None
        self.lin = IrrepsLinear(self.dtp.irreps_out.simplify(), irreps_lin_out)

    def tp(self, x, sh, edge_scalars):
        return self.dtp(x, sh) if self.rad is None else self.dtp(x, sh, self.rad(edge_scalars))

    def forward(self, x, sh, edge_scalars):
        return self.lin(self.tp(x, sh, edge_scalars))


class MLPAttentionScores(nn.Module):
    def __init__(self, num_heads: int, mul_alpha_head: int):
        super().__init__()
        self.alpha_act = SmoothLeakyReLU(0.2)
        self.alpha_scale = moment_scale(SmoothLeakyReLU(0.2))
        bound = math.sqrt(6.0 / (num_heads + mul_alpha_head))
        self.alpha_dot = nn.Parameter(torch.empty(1, num_heads, mul_alpha_head).uniform_(-bound, bound))

    def forward(self, alpha: Tensor) -> Tensor:
        return torch.einsum("ehk,hk->eh", self.alpha_act(alpha) * self.alpha_scale, self.alpha_dot[0])


class NonlinearMLPAttention(nn.Module):
    def __init__(self, pre, irreps_sh, attn_heads, irreps_alpha, radial, heads: Heads, num_heads: int,
                 mul_alpha_head: int):
        super().__init__()
        self.num_heads, self.mul_alpha_head = num_heads, mul_alpha_head
        gate = Gate(pre)
        self.sep_act = SeparableTP(pre, irreps_sh, pre, gate.irreps_in, radial)
        self.gate = gate
        self.sep_alpha = IrrepsLinear(self.sep_act.dtp.irreps_out.simplify(), irreps_alpha)
        self.sep_value = SeparableTP(pre, irreps_sh, attn_heads, attn_heads, None)
        self.scores = MLPAttentionScores(num_heads, mul_alpha_head)
        self.heads = heads

    def forward(self, x, msg, dst, sh, edge_scalars):
        f = self.sep_act.tp(msg, sh, edge_scalars)
        alpha = self.sep_alpha(f).reshape(f.shape[0], self.num_heads, self.mul_alpha_head)
        value = self.heads.split(self.sep_value(self.gate(self.sep_act.lin(f)), sh, edge_scalars))
        return self.scores(alpha), value


class LinearMLPAttention(nn.Module):
    def __init__(self, pre, irreps_sh, attn_heads, irreps_alpha, irreps_head, radial, num_heads: int,
                 mul_alpha_head: int):
        super().__init__()
        self.mul_alpha_head = mul_alpha_head
        attn_all = (irreps_alpha + attn_heads).simplify()
        self.sep = SeparableTP(pre, irreps_sh, attn_all, attn_all, radial)
        self.heads_all = Heads((Irreps(f"{mul_alpha_head}x0e") + irreps_head).simplify(), num_heads)
        self.scores = MLPAttentionScores(num_heads, mul_alpha_head)

    def forward(self, x, msg, dst, sh, edge_scalars):
        f = self.heads_all.split(self.sep(msg, sh, edge_scalars))
        return self.scores(f[:, :, :self.mul_alpha_head]), f[:, :, self.mul_alpha_head:]


class DotProductAttention(nn.Module):
    def __init__(self, irreps_in, pre, irreps_sh, attn_heads, irreps_head, radial, heads: Heads, num_heads: int):
        super().__init__()
        self.num_heads = num_heads
        self.query = IrrepsLinear(irreps_in, attn_heads)
        kv = sort_irreps(irreps_head * (2 * num_heads), even_first=False)
        self.key_value = SeparableTP(pre, irreps_sh, kv, kv, radial)
        self.heads, self.heads_kv = heads, Heads(irreps_head, 2 * num_heads)
        scale = [1.0 / math.sqrt(irreps_head.num_irreps * ir.dim) for mul, ir in irreps_head for _ in range(mul * ir.dim)]
        self.register_buffer("q_scale", torch.tensor(scale), persistent=False)

    def forward(self, x, msg, dst, sh, edge_scalars):
        q = self.heads.split(self.query(x)) * self.q_scale
        kv = self.heads_kv.split(self.key_value(msg, sh, edge_scalars))
        return (q[dst] * kv[:, :self.num_heads]).sum(-1), kv[:, self.num_heads:2 * self.num_heads]


class GraphAttention(nn.Module):
    def __init__(self, irreps_in, irreps_sh, irreps_out, radial, irreps_head, num_heads: int, irreps_pre_attn=None,
                 attention: str = "mlp", nonlinear_message: bool = True, rescale_degree: bool = False,
                 alpha_drop: float = 0.0, proj_drop: float = 0.0, avg_degree: float = AVG_DEGREE):
        super().__init__()
        if attention not in ("mlp", "dot_product"):
            raise ValueError(f"attention must be 'mlp' or 'dot_product', got {attention!r}")
        irreps_in, irreps_head = Irreps(irreps_in), Irreps(irreps_head)
        pre = irreps_in if irreps_pre_attn is None else Irreps(irreps_pre_attn)
        mlp = attention == "mlp"
        self.rescale_degree = bool(rescale_degree)
        self.degree_divisor = 1.0 if mlp else float(avg_degree)
        attn_heads = sort_irreps(irreps_head * num_heads, even_first=mlp)
        self.merge_src = IrrepsLinear(irreps_in, pre, bias=True)
        self.merge_dst = IrrepsLinear(irreps_in, pre, bias=False)
        self.heads = Heads(irreps_head, num_heads)
        if mlp:
            mul_alpha = sum(mul for mul, ir in attn_heads if ir == Irrep(0, 1))
            alpha = Irreps(f"{mul_alpha}x0e")
            self.core = (NonlinearMLPAttention(pre, irreps_sh, attn_heads, alpha, radial, self.heads, num_heads,
                                               mul_alpha // num_heads) if nonlinear_message else
                         LinearMLPAttention(pre, irreps_sh, attn_heads, alpha, irreps_head, radial, num_heads,
                                            mul_alpha // num_heads))
        else:
            self.core = DotProductAttention(irreps_in, pre, irreps_sh, attn_heads, irreps_head, radial, self.heads,
                                            num_heads)
        self.alpha_dropout = nn.Dropout(alpha_drop) if alpha_drop > 0 else nn.Identity()
        self.proj = IrrepsLinear(attn_heads, irreps_out)
        self.proj_drop = ChannelDropout(irreps_in, proj_drop)

    def forward(self, x, src, dst, sh, edge_scalars, envelope: Optional[Tensor]):
        n = x.shape[0]
        msg = self.merge_src(x)[src] + self.merge_dst(x)[dst]
        logits, value = self.core(x, msg, dst, sh, edge_scalars)
        attn = self.alpha_dropout(segment_softmax(logits, dst, n, envelope))
        out = self.heads.merge(scatter_sum(value * attn.unsqueeze(-1), dst, n))
        if self.rescale_degree:
            out = out * scatter_sum(torch.ones_like(dst, dtype=out.dtype), dst, n).unsqueeze(-1) / self.degree_divisor
        return self.proj_drop(self.proj(out))


class FeedForward(nn.Module):
    def __init__(self, irreps_in, irreps_mid, irreps_out, proj_drop: float = 0.0):
        super().__init__()
        self.gate = Gate(irreps_mid)
        self.lin_1 = IrrepsLinear(irreps_in, self.gate.irreps_in)
        self.lin_2 = IrrepsLinear(self.gate.irreps_out, irreps_out)
        self.proj_drop = ChannelDropout(irreps_out, proj_drop)

    def forward(self, x):
        return self.proj_drop(self.lin_2(self.gate(self.lin_1(x))))


class TransformerBlock(nn.Module):
    def __init__(self, irreps_in, irreps_sh, irreps_out, radial, irreps_head, num_heads, irreps_pre_attn,
                 irreps_mlp_mid, attention, nonlinear_message, rescale_degree, alpha_drop, proj_drop, drop_path_rate,
                 avg_degree):
        super().__init__()
        irreps_in, irreps_out = Irreps(irreps_in), Irreps(irreps_out)
        self.norm_1 = EquivariantLayerNorm(irreps_in)
        self.ga = GraphAttention(irreps_in, irreps_sh, irreps_in, radial, irreps_head, num_heads, irreps_pre_attn,
                                 attention, nonlinear_message, rescale_degree, alpha_drop, proj_drop, avg_degree)
        self.drop_path = GraphDropPath(drop_path_rate)
        self.norm_2 = EquivariantLayerNorm(irreps_in)
        self.ffn = FeedForward(irreps_in, irreps_mlp_mid, irreps_out, proj_drop)
        self.ffn_shortcut = IrrepsLinear(irreps_in, irreps_out) if irreps_in != irreps_out else None

    def forward(self, x, src, dst, sh, edge_scalars, envelope, batch, num_graphs: int):
        x = x + self.drop_path(self.ga(self.norm_1(x), src, dst, sh, edge_scalars, envelope), batch, num_graphs)
        h = self.ffn(self.norm_2(x))
        if self.ffn_shortcut is not None:
            x = self.ffn_shortcut(x)
        return x + self.drop_path(h, batch, num_graphs)


class EdgeDegreeEmbedding(nn.Module):
    def __init__(self, irreps_node, irreps_sh, radial, avg_degree: float):
        super().__init__()
        self.exp = IrrepsLinear("1x0e", irreps_node)
        self.dw = depthwise_tensor_product(irreps_node, irreps_sh, irreps_node, internal_weights=False)
        self.rad = RadialMLP(radial + [self.dw.weight_numel])
        self.proj = IrrepsLinear(self.dw.irreps_out.simplify(), irreps_node)
        self.avg_degree = float(avg_degree)

    def forward(self, n: int, sh, edge_scalars, dst, envelope: Optional[Tensor]):
        const = self.exp(sh.new_ones((1, 1))).expand(sh.shape[0], -1)
        edge = self.proj(self.dw(const, sh, self.rad(edge_scalars)))
        if envelope is not None:
            edge = edge * envelope.unsqueeze(-1)
        return scatter_sum(edge, dst, n) / math.sqrt(self.avg_degree)


class AtomEmbedding(nn.Module):
    def __init__(self, n_elements: int, irreps_node):
        super().__init__()
        irreps_node = Irreps(irreps_node)
        if irreps_node[0][1] != Irrep(0, 1):
            raise ValueError(f"the node irreps must start with even scalars, got {irreps_node}")
        self.n_scalars, self.n_rest = irreps_node[0].mul, irreps_node.dim - irreps_node[0].mul
        self.weight = nn.Parameter(torch.randn(n_elements, self.n_scalars))
        self.bias = nn.Parameter(torch.zeros(self.n_scalars))

    def forward(self, z: Tensor) -> Tensor:
        s = self.weight[z] + self.bias
        return torch.cat([s, s.new_zeros((s.shape[0], self.n_rest))], 1)


@register_model("equiformer")
class Equiformer(TransformerPotential):
    head_modules = ("head", "energy_scale", "energy_shift", "atom_ref")

    def __init__(self, irreps_node_embedding: str = "128x0e+64x1e+32x2e", n_interactions: int = 6, cutoff: float = 5.0,
                 n_rbf: int = 32, radial_basis: str = "expnorm", radial_hidden: Optional[List[int]] = None,
                 irreps_sh: Optional[str] = None, irreps_feature: str = "512x0e", irreps_head: str = "32x0e+16x1e+8x2e",
                 num_heads: int = 4, irreps_pre_attn: Optional[str] = None,
                 irreps_mlp_mid: str = "384x0e+192x1e+96x2e", attention: str = "mlp", nonlinear_message: bool = True,
                 rescale_degree: bool = False, alpha_drop: float = 0.0, proj_drop: float = 0.0, out_drop: float = 0.0,
                 drop_path_rate: float = 0.0, avg_degree: float = AVG_DEGREE, avg_num_nodes: float = AVG_NUM_NODES,
                 smooth_cutoff: bool = False, n_elements: int = 100, energy_shift: float = 0.0,
                 energy_scale: float = 1.0, species=None, atomic_energies=None):
        super().__init__()
        self.cutoff = float(cutoff)
        if species is not None:
            self.species = [int(z) for z in species]
        self.irreps_node_embedding, self.irreps_feature = Irreps(irreps_node_embedding), Irreps(irreps_feature)
        if irreps_sh is None:
            lmax = self.irreps_node_embedding.lmax
            irreps_sh = ("+".join(f"1x{l}e" for l in range(lmax + 1)) if all(ir.p == 1 for _, ir in self.irreps_node_embedding)
                         else str(Irreps.spherical_harmonics(lmax)))
        self.irreps_sh = Irreps(irreps_sh)
        self.n_interactions, self.avg_num_nodes, self.smooth = n_interactions, float(avg_num_nodes), bool(smooth_cutoff)
        self.node_feature_dim = sum(mul for mul, ir in self.irreps_feature if ir == Irrep(0, 1))
        radial = [n_rbf] + list(radial_hidden if radial_hidden is not None else [64, 64])
        self.sh = SphericalHarmonics(self.irreps_sh, normalize=True, normalization="component")
        self.rbf = make_radial_basis(radial_basis, n_rbf, cutoff)
        self.envelope = PolynomialCutoff(cutoff, p=6)
        self.atom_embed = AtomEmbedding(n_elements, self.irreps_node_embedding)
        self.edge_deg_embed = EdgeDegreeEmbedding(self.irreps_node_embedding, self.irreps_sh, radial, avg_degree)
        self.blocks = nn.ModuleList(TransformerBlock(
            self.irreps_node_embedding, self.irreps_sh,
            self.irreps_feature if k == n_interactions - 1 else self.irreps_node_embedding, radial, irreps_head,
            num_heads, irreps_pre_attn, irreps_mlp_mid, attention, nonlinear_message, rescale_degree, alpha_drop,
            proj_drop, drop_path_rate, avg_degree) for k in range(n_interactions))
        self.norm = EquivariantLayerNorm(self.irreps_feature)
        self.out_dropout = ChannelDropout(self.irreps_feature, out_drop)
        gate = Gate(self.irreps_feature)
        self.head = nn.ModuleList([IrrepsLinear(self.irreps_feature, gate.irreps_in), gate,
                                   IrrepsLinear(gate.irreps_out, "1x0e")])
        self._init_energy_terms(n_elements, energy_scale, energy_shift, species, atomic_energies)

    def receptive_field(self):
        return self.n_interactions * self.cutoff

    def _evaluate(self, z, edge_index, edge_vec, batch, num_graphs: int):
        n = z.shape[0]
        src, dst = edge_index[0], edge_index[1]
        r = torch.linalg.norm(edge_vec, dim=-1)
        sh = self.sh(-edge_vec)
        edge_scalars = self.rbf(r)
        envelope = self.envelope(r) if self.smooth else None
        x = self.atom_embed(z) + self.edge_deg_embed(n, sh, edge_scalars, dst, envelope)
        for block in self.blocks:
            x = block(x, src, dst, sh, edge_scalars, envelope, batch, num_graphs)
        x = self.out_dropout(self.norm(x))
        y = x
        for layer in self.head:
            y = layer(y)
        return x, y.squeeze(-1) / math.sqrt(self.avg_num_nodes)

    def _energy(self, y, z):
        return self.energy_scale * y + self.energy_shift + self.atom_ref(z).squeeze(-1)

    def node_features_energy(self, atomic_numbers, edge_index, edge_vec):
        x, y = self._evaluate(atomic_numbers, edge_index, edge_vec, torch.zeros_like(atomic_numbers), 1)
        return x[:, :self.node_feature_dim], self._energy(y, atomic_numbers)

    def forward(self, data: AtomicGraph) -> Dict[str, Tensor]:
        x, y = self._evaluate(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.batch, data.num_graphs)
        node = self._energy(y, data.atomic_numbers)
        return {"node_energy": node, "energy": self.aggregate_energy(node, data), "node_features": x[:, :self.node_feature_dim]}

    @classmethod
    def from_config(cls, cfg) -> "Equiformer":
        e = dict(cfg.extra or {})
        preset = paper_irreps(int(e.get("l_max", 2)), bool(e.get("e3", False)), int(cfg.n_features))
        kw = {k: e.get(k, v) for k, v in preset.items()}
        for key in ("irreps_sh", "irreps_feature", "irreps_pre_attn", "radial_hidden", "radial_basis", "attention",
                    "nonlinear_message", "rescale_degree", "smooth_cutoff", "alpha_drop", "proj_drop", "out_drop",
                    "drop_path_rate", "avg_degree", "avg_num_nodes", "n_elements", "energy_shift", "energy_scale",
                    "species", "atomic_energies"):
            if e.get(key) is not None:
                kw[key] = e[key]
        if kw.get("radial_basis") == "exp":
            kw["radial_basis"] = "expnorm"
        kw["num_heads"] = int(kw["num_heads"])
        return cls(n_interactions=cfg.n_interactions, cutoff=cfg.cutoff, n_rbf=cfg.n_rbf, **kw)
