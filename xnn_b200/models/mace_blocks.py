"""The MACE coupling basis and symmetric contraction (reference path).

``U_matrix_real`` couples ``correlation`` copies of the input irreps into each output
irrep as a left fold: the paths of the first ``d`` factors are extended with a
Wigner 3j symbol against every irrep of factor ``d + 1``, and the path list is sorted
(stably) by coupled irrep after every stage; the paths that reach an output irrep are
stacked along a trailing axis. The enumeration order fixes the layout of the learned
weights, so it follows the reference (``src/xnn/gnn/models/mace.py:68-215``), which is
itself bit-compatible with mace-torch.

``SymmetricContraction`` evaluates ``sum_nu sum_k W_nu[z, k, c] U_nu[..., k] x^nu`` per
channel ``c`` and element ``z`` (MACE Eq. 10-11; ``mace.py:244-564``), Horner style
from the highest order down.
"""
from __future__ import annotations

import functools
from typing import List, Optional, Tuple

import torch
from torch import Tensor, nn

from ..o3 import Irrep, Irreps, wigner_3j


def _couple_paths(factors: List[Irreps], normalization: str = "component",
                  keep=None, dtype=None) -> List[Tuple[Irrep, Tensor]]:
    """Every coupling path of one irrep from each factor into a single irrep."""
    first = factors[0]
    eye = torch.eye(first.dim, dtype=dtype)
    paths: List[Tuple[Irrep, Tensor]] = []
    row = 0
    for mul, ir in first:
        for _ in range(mul):
            paths.append((ir, eye[row:row + ir.dim]))
            row += ir.dim
    for depth in range(1, len(factors)):
        fac = factors[depth]
        lead = [f.dim for f in factors[:depth]]
        grown: List[Tuple[Irrep, Tensor]] = []
        for ir_acc, w_acc in paths:
            col = 0
            for mul, ir_f in fac:
                for ir_tot in ir_acc * ir_f:
                    if keep is not None and ir_tot not in keep:
                        continue
                    c3 = wigner_3j(ir_tot.l, ir_acc.l, ir_f.l, dtype=dtype)
                    if normalization == "component":
                        c3 = c3 * ir_tot.dim ** 0.5
                    elif normalization == "norm":
                        c3 = c3 * (ir_acc.dim ** 0.5 * ir_f.dim ** 0.5)
                    coupled = torch.einsum("ap,oaf->opf", w_acc.flatten(1), c3)
                    coupled = coupled.reshape(ir_tot.dim, *lead, ir_f.dim)
                    for copy in range(mul):
                        lo = col + copy * ir_f.dim
                        emb = torch.zeros(ir_tot.dim, *lead, fac.dim, dtype=dtype)
                        emb[..., lo:lo + ir_f.dim] = coupled
                        grown.append((ir_tot, emb))
                col += mul * ir_f.dim
        grown.sort(key=lambda e: e[0])  # stable: ties keep enumeration order
        paths = grown
    return paths


def U_matrix_real(irreps_in, irreps_out, correlation: int, normalization: str = "component",
                  filter_ir_mid=None, dtype=None) -> list:
    """``[ir, U, ir, U, ...]``: per output irrep the stacked coupling paths ``(..., n_paths)``."""
    irreps_out = Irreps(irreps_out)
    if correlation == 4:
        filter_ir_mid = [Irrep(l, (-1) ** l) for l in range(12)]
    keep = None if filter_ir_mid is None else frozenset(Irrep(i) for i in filter_ir_mid)
    paths = _couple_paths([Irreps(irreps_in)] * correlation, normalization, keep, dtype)
    out: list = []
    i = 0
    while i < len(paths):
        ir = paths[i][0]
        j = i
        while j < len(paths) and paths[j][0] == ir:
            j += 1
        if ir in irreps_out:
            out.append(ir)
            out.append(torch.stack([w.squeeze() for _, w in paths[i:j]], dim=-1))
        i = j
    if out:
        return out
    shape = [Irreps(irreps_in).dim] * correlation + [1]
    if irreps_out.dim != 1:
        shape.insert(0, irreps_out.dim)
    text = str(irreps_out)
    return [text[:len(text) - 2], torch.zeros(shape, dtype=dtype)]


@functools.lru_cache(maxsize=None)
def exact_U(irreps_in: str, irrep_out: str, nu: int) -> Tensor:
    return U_matrix_real(Irreps(irreps_in), Irreps(irrep_out), nu, dtype=torch.float64)[-1]


class Contraction(nn.Module):
    """The per-output-irrep piece of the symmetric contraction (one ``U_matrix_nu`` per order)."""

    def __init__(self, irreps_in, irrep_out, correlation: int, num_elements: int):
        super().__init__()
        if not 1 <= correlation <= 4:
            raise NotImplementedError(f"correlation={correlation} is outside 1..4")
        irreps_in = Irreps(irreps_in)
        self.num_features = irreps_in.count("0e")
        self.coupling_irreps = Irreps([m.ir for m in irreps_in])
        self.correlation = correlation
        self.irrep_out = Irreps(irrep_out)
        self.lmax_out = self.irrep_out.lmax
        dtype = torch.get_default_dtype()
        for nu in range(1, correlation + 1):
            U = U_matrix_real(self.coupling_irreps, self.irrep_out, nu, dtype=torch.float64)[-1]
            self.register_buffer(f"U_matrix_{nu}", U.to(dtype))
        for nu in range(correlation + 1, 5):
            self.register_buffer(f"U_matrix_{nu}", torch.zeros(0, dtype=dtype), persistent=False)
        self.weights = nn.ParameterList()
        for nu in range(1, correlation + 1):
            k = self.U(nu).shape[-1]
            self.weights.append(nn.Parameter(torch.randn(num_elements, k, self.num_features) / k))

    def U(self, nu: int) -> Tensor:
        return getattr(self, f"U_matrix_{nu}")

    def forward(self, x: Tensor, y: Tensor) -> Tensor:
        """``x (B, C, dim)`` features, ``y (B, n_el)`` one-hot elements -> ``(B, C * out_dim)``."""
        B, C, dim = x.shape
        n_el = y.shape[1]
        m_out = 2 * self.lmax_out + 1 if self.lmax_out > 0 else 1
        xt = x.transpose(0, 1)                      # (C, B, dim)
        corr = self.correlation
        U = self.U(corr)
        K = U.shape[-1]
        W = self.weights[corr - 1]                  # (n_el, K, C)
        # (C, n_el, M * dim^(corr-1), dim) with the last coupling index split off
        uw = torch.einsum("xk,ekc->cex", U.reshape(-1, K), W)
        uw = uw.reshape(C, n_el, -1, dim).transpose(2, 3).reshape(C, n_el * dim, -1)
        outer = (y[None, :, :, None] * xt[:, :, None, :]).reshape(C, B, n_el * dim)
        acc = torch.bmm(outer, uw)                  # (C, B, M * dim^(corr-1))
        for nu in range(corr - 1, 0, -1):
            U = self.U(nu)
            K = U.shape[-1]
            W = self.weights[nu - 1]
            w_el = torch.einsum("xk,ekc->ecx", U.reshape(-1, K), W).reshape(n_el, -1)
            weighted = (y @ w_el).reshape(B, C, -1).transpose(0, 1)
            acc = acc + weighted
            acc = (acc.reshape(C, B, -1, dim) * xt[:, :, None, :]).sum(-1)
        return acc.reshape(C, B, m_out).transpose(0, 1).reshape(B, C * m_out)


class SymmetricContraction(nn.Module):
    def __init__(self, irreps_in, irreps_out, correlation: int, num_elements: int):
        super().__init__()
        self.irreps_in = Irreps(irreps_in)
        self.irreps_out = Irreps(irreps_out)
        self.contractions = nn.ModuleList([
            Contraction(self.irreps_in, Irreps(str(m.ir)), correlation, num_elements)
            for m in self.irreps_out])

    def forward(self, x: Tensor, y: Tensor) -> Tensor:
        return torch.cat([c(x, y) for c in self.contractions], dim=-1)


def tp_out_irreps_with_instructions(irreps1, irreps2, target_irreps, sort_instructions: bool = True):
    """``uvu`` paths of ``irreps1 x irreps2`` landing in ``target_irreps``, outputs sorted
    (``src/xnn/gnn/models/blocks.py:77-115``)."""
    wanted = Irreps(target_irreps)
    kept = []
    paths = []
    for a, (mul, ir_a) in enumerate(Irreps(irreps1)):
        for b, (_, ir_b) in enumerate(Irreps(irreps2)):
            for ir in ir_a * ir_b:
                if ir in wanted:
                    paths.append((a, b, len(kept), "uvu", True))
                    kept.append((mul, ir))
    sorted_irreps, remap, _ = Irreps(kept).sort()
    paths = [(a, b, remap[s], m, w) for a, b, s, m, w in paths]
    if sort_instructions:
        paths.sort(key=lambda p: p[2])
    return sorted_irreps, paths


def hidden_irreps(mul: int, lmax: int) -> Irreps:
    return Irreps([(mul, m.ir) for m in Irreps.spherical_harmonics(lmax)])


class ReshapeIrreps(nn.Module):
    """Flat ``(N, irreps.dim)`` -> ``(N, mul, sum of ir dims)`` (uniform multiplicity)."""

    def __init__(self, irreps):
        super().__init__()
        self.irreps = Irreps(irreps)

    def forward(self, t: Tensor) -> Tensor:
        out, i = [], 0
        for mul, ir in self.irreps:
            d = mul * ir.dim
            out.append(t[:, i:i + d].reshape(-1, mul, ir.dim))
            i += d
        return torch.cat(out, dim=-1)
