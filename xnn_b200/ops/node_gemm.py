"""Batched node-level products of the MACE training step (``csrc/node_gemm.cu``).

A problem table goes to one kernel launch:

* :class:`MM` -- ``Y[rows] (+)= [X0 | X1][rows] @ W``; rows optionally gathered / scattered
  through ``perm`` and restricted to the segment ``seg = (start, end)`` of the permuted row
  space (device tensor, e.g. the atoms of one element);
* :class:`MMT` -- ``out = scale * (X0^T D0 + X1^T D1)`` summed over the rows (same row
  options), split over CTAs whose partial blocks a second kernel sums in a fixed order
  (deterministic).

Weights are packed once per step (:func:`pack`) into the MMA operand layout. On the CPU (and
for shapes the kernel does not take) the same problems evaluate with PyTorch, which is what the
tests compare against.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch
from torch import Tensor

from .. import _ext

SPIN_LIMIT = 50_000_000
#: atoms up to which the one-CTA species sort kernel is used (it serves the training batches)
SORT_KERNEL_MAX = 65536
_STATE: Dict[torch.device, Dict[str, Tensor]] = {}


def _state(dev: torch.device) -> Dict[str, Tensor]:
    st = _STATE.get(dev)
    if st is None:
        st = {"status": torch.zeros(1, dtype=torch.int32, device=dev),
              "counters": torch.zeros(64, dtype=torch.int32, device=dev)}
        _STATE[dev] = st
    return st


def status(dev: torch.device) -> int:
    """Non-zero when a node product on ``dev`` gave up waiting (reading it synchronises)."""
    st = _STATE.get(dev)
    return 0 if st is None else int(st["status"].item())


def kernels(t: Tensor) -> bool:
    return t.is_cuda and t.dtype == torch.float32 and _ext.cuda_available()


@dataclass
class MM:
    X0: Tensor
    W: object                      # (K0 + K1, N) unpacked, or a pair (upper, lower) of row blocks
    Y: Tensor
    Wp: Optional[Tensor] = None    # packed W (CUDA)
    X1: Optional[Tensor] = None
    perm: Optional[Tensor] = None  # int32 (CUDA) / int64 (CPU) permutation of the rows
    seg: Optional[Tensor] = None   # two-entry tensor: the problem's rows [seg[0], seg[1])
    rows: Optional[int] = None     # row count (default: X0 rows); with seg an upper bound
    accumulate: bool = False


@dataclass
class MMT:
    X0: Tensor
    D0: Tensor
    out: Tensor
    X1: Optional[Tensor] = None
    D1: Optional[Tensor] = None
    perm: Optional[Tensor] = None
    seg: Optional[Tensor] = None
    rows0: Optional[int] = None
    rows1: Optional[int] = None
    scale: float = 1.0


def pack(Ws: Sequence) -> List[Tensor]:
    """Packed operand copies of the float32 CUDA matrices ``Ws`` (one launch per 48; any strides,
    so transposed views need no copy). An entry ``(A, B)`` packs ``A`` stacked above ``B``."""
    out: List[Tensor] = []
    Ws = list(Ws)
    for i in range(0, len(Ws), 48):
        chunk = Ws[i:i + 48]
        top = [w[0] if isinstance(w, tuple) else w for w in chunk]
        low = [w[1] if isinstance(w, tuple) else None for w in chunk]
        out += _ext.ops().node_pack(top, low)
    return out


def _rows_of(p_rows: Optional[int], X: Tensor, seg: Optional[Tensor], perm: Optional[Tensor]) -> Tensor:
    n = X.shape[0] if p_rows is None else int(p_rows)
    if seg is not None:
        s = seg.tolist()
        idx = torch.arange(int(s[0]), int(s[1]), device=X.device)
    else:
        idx = torch.arange(n, device=X.device)
    return perm.long()[idx] if perm is not None else idx


def _mm_torch(p: MM) -> None:
    idx = _rows_of(p.rows, p.X0, p.seg, p.perm)
    x = p.X0.index_select(0, idx)
    if p.X1 is not None:
        x = torch.cat([x, p.X1.index_select(0, idx)], 1)
    W = torch.cat(p.W, 0) if isinstance(p.W, tuple) else p.W
    y = x @ W.to(x.dtype)
    if p.accumulate:
        p.Y.index_add_(0, idx, y)
    else:
        p.Y.index_copy_(0, idx, y)


def _mmt_torch(p: MMT) -> None:
    idx = _rows_of(p.rows0, p.X0, p.seg, p.perm)
    g = p.X0.index_select(0, idx).t() @ p.D0.index_select(0, idx)
    if p.X1 is not None:
        idx1 = _rows_of(p.rows1, p.X1, p.seg, p.perm)
        g = g + p.X1.index_select(0, idx1).t() @ p.D1.index_select(0, idx1)
    p.out.copy_((p.scale * g).view_as(p.out))


def _mm_ok(p: MM) -> bool:
    N = p.Y.shape[1]
    K = p.X0.shape[1] + (0 if p.X1 is None else p.X1.shape[1])
    return (kernels(p.X0) and p.Wp is not None and 16 <= N <= 128 and N % 16 == 0 and p.X0.shape[1] % 4 == 0
            and (p.X1 is None or p.X1.shape[1] % 4 == 0) and K == _w_rows(p.W))


def _w_rows(W) -> int:
    return sum(int(w.shape[0]) for w in W) if isinstance(W, tuple) else int(W.shape[0])


def _mmt_ok(p: MMT) -> bool:
    K1, N = p.X0.shape[1], p.D0.shape[1]
    return kernels(p.X0) and K1 % 4 == 0 and 4 <= K1 <= 128 and N % 16 == 0 and 16 <= N <= 256


def mm(problems: Sequence[MM], trace: Optional[Tensor] = None) -> None:
    """Run every row product (one kernel launch for those the kernel takes). ``trace`` (int64,
    8 slots per CTA) receives each CTA's phase timestamps in nanoseconds (diagnostics)."""
    fast = [p for p in problems if _mm_ok(p)]
    for p in problems:
        if not _mm_ok(p):
            _mm_torch(p)
    if not fast:
        return
    st = _state(fast[0].X0.device)
    for i in range(0, len(fast), 24):
        chunk = fast[i:i + 24]
        _ext.ops().node_mm([p.X0 for p in chunk], [p.X1 for p in chunk], [p.Y for p in chunk],
                           [p.Wp for p in chunk], [p.perm for p in chunk], [p.seg for p in chunk],
                           [int(p.X0.shape[0] if p.rows is None else p.rows) for p in chunk],
                           [bool(p.accumulate) for p in chunk], st["status"], SPIN_LIMIT, trace)


def mmT(problems: Sequence[MMT], trace: Optional[Tensor] = None) -> None:
    """Run every reduction (one kernel launch for those the kernel takes); ``trace`` as in
    :func:`mm`."""
    fast = [p for p in problems if _mmt_ok(p)]
    for p in problems:
        if not _mmt_ok(p):
            _mmt_torch(p)
    if not fast:
        return
    st = _state(fast[0].X0.device)
    for i in range(0, len(fast), 16):
        chunk = fast[i:i + 16]
        _ext.ops().node_mmT([p.X0 for p in chunk], [p.D0 for p in chunk], [p.X1 for p in chunk],
                            [p.D1 for p in chunk], [p.perm for p in chunk], [p.seg for p in chunk],
                            [int(p.X0.shape[0] if p.rows0 is None else p.rows0) for p in chunk],
                            [int(0 if p.X1 is None else (p.X1.shape[0] if p.rows1 is None else p.rows1))
                             for p in chunk],
                            [p.out for p in chunk], [float(p.scale) for p in chunk], st["counters"],
                            st["status"], SPIN_LIMIT, trace)


def species_sort(z: Tensor, n_el: int):
    """``(perm, seg)``: atoms grouped by element index (stable), element ``k`` at
    ``perm[seg[k]:seg[k + 1]]``; int32 on CUDA."""
    if z.is_cuda and _ext.cuda_available() and z.numel() <= SORT_KERNEL_MAX:
        return _ext.ops().species_sort(z.contiguous(), int(n_el))
    if z.is_cuda:                  # large systems: the library's radix sort (the kernel is one CTA)
        perm = torch.argsort(z, stable=True).to(torch.int32)
        seg = torch.zeros(n_el + 1, dtype=torch.int32, device=z.device)
        seg[1:] = torch.cumsum(torch.bincount(z, minlength=n_el), 0).to(torch.int32)
        return perm, seg
    perm = torch.argsort(z, stable=True)
    counts = torch.bincount(z, minlength=n_el)
    seg = torch.zeros(n_el + 1, dtype=torch.long, device=z.device)
    seg[1:] = torch.cumsum(counts, 0)
    return perm, seg


def segment_sum(X: Tensor, perm: Tensor, seg: Tensor, z: Tensor, groups: int) -> Tensor:
    """Row sums of ``X`` per group: ``out[k] = sum_{i: z_i = k} X[i]`` (``perm, seg`` from
    :func:`species_sort` of ``z``); one fixed-order kernel on CUDA."""
    if X.is_cuda and X.dtype in (torch.float32, torch.float64) and _ext.cuda_available():
        return _ext.ops().segment_rows_sum(X.contiguous(), perm, seg)
    return X.new_zeros((groups,) + tuple(X.shape[1:])).index_add_(0, z, X)


def edge_forces(plan, v: Tensor, out_dtype: torch.dtype) -> Tensor:
    """``F_i = sum_{e: src=i} v_e - sum_{e: dst=i} v_e`` for per-edge vectors ``v (E, 3)`` through the
    plan's CSR orderings (one fixed-order kernel on CUDA), in ``out_dtype``."""
    if v.is_cuda and _ext.cuda_available():
        return _ext.ops().edge_forces(plan.dst_ptr, plan.dst_perm, plan.src_ptr, plan.src_perm, v.contiguous(),
                                      out_dtype)
    F = torch.zeros(plan.n_nodes, 3, dtype=v.dtype, device=v.device)
    return F.index_add_(0, plan.src, v).index_add_(0, plan.dst, -v).to(out_dtype)


def _grouped_rows(z: Tensor, n_el: int, lead: int):
    """Row permutation and element segments of ``lead`` stacked copies of the atoms: element
    ``k``'s rows (every copy) are ``perm[lead * seg[k]:lead * seg[k + 1]]``; plus the host counts."""
    perm, seg = species_sort(z, n_el)
    N = z.shape[0]
    seg64 = seg.long()
    segs = (seg64 * lead).to(torch.int32)
    if lead == 1:
        return perm, segs, seg64.cpu()
    q = torch.arange(lead * N, device=z.device)
    k = torch.searchsorted(segs[1:].long(), q, right=True)
    s, c = seg64[k], (seg64[k + 1] - seg64[k]).clamp_min(1)
    local = q - lead * s
    full = (local // c) * N + perm.long()[s + local % c]
    return full.to(torch.int32), segs, seg64.cpu()


def _grouped_product(X: Tensor, Ws: Sequence[Tensor], perm: Tensor, segs: Tensor, counts: Tensor,
                     lead: int) -> Tensor:
    Y = torch.empty(X.shape[0], Ws[0].shape[1], dtype=X.dtype, device=X.device)
    packed = pack(list(Ws))
    probs = []
    for k, W in enumerate(Ws):
        rows = lead * int(counts[k + 1] - counts[k])
        if rows > 0:
            probs.append(MM(X, W, Y, packed[k], perm=perm, seg=segs[k:k + 2], rows=rows))
    mm(probs)
    return Y


class _SpeciesLinear(torch.autograd.Function):
    """``Y = X @ W[z]`` per row, rows grouped by element; the backward is the same product with
    the transposed matrices (differentiable again). The weights are constants here."""

    @staticmethod
    def forward(ctx, X: Tensor, Wz: Tensor, perm: Tensor, segs: Tensor, counts: Tensor, lead: int):
        ctx.save_for_backward(Wz, perm, segs)
        ctx.counts, ctx.lead = counts, lead
        return _grouped_product(X, list(Wz.unbind(0)), perm, segs, counts, lead)

    @staticmethod
    def backward(ctx, g: Tensor):
        Wz, perm, segs = ctx.saved_tensors
        dX = _SpeciesLinear.apply(g.contiguous(), Wz.transpose(1, 2), perm, segs, ctx.counts, ctx.lead)
        return dX, None, None, None, None, None


def grouped_species_ok(h: Tensor, Wz: Tensor) -> bool:
    """Whether :func:`species_linear` takes the grouped kernel for these operands."""
    c_in, c_out = int(Wz.shape[1]), int(Wz.shape[2])
    ok = lambda n: 16 <= n <= 128 and n % 16 == 0
    return (kernels(h) and Wz.dtype == torch.float32 and ok(c_in) and ok(c_out) and h.shape[-1] == c_in
            and not torch.cuda.is_current_stream_capturing())      # it reads the element counts


class _SpeciesLinearBlocks(torch.autograd.Function):
    """``Y = X @ W_l[z]`` for rows of ``lead`` stacked components split into per-degree blocks of
    ``sizes`` components each (one matrix per element and block); the weights are constants."""

    @staticmethod
    def forward(ctx, X: Tensor, Ws: Tensor, perm: Tensor, segs: Tensor, counts: Tensor, sizes: Tuple[int, ...]):
        ctx.save_for_backward(Ws, perm, segs)
        ctx.counts, ctx.sizes = counts, sizes
        return _blocks_product(X, Ws, perm, segs, counts, sizes)

    @staticmethod
    def backward(ctx, g: Tensor):
        Ws, perm, segs = ctx.saved_tensors
        dX = _SpeciesLinearBlocks.apply(g.contiguous(), Ws.transpose(-1, -2), perm, segs, ctx.counts, ctx.sizes)
        return dX, None, None, None, None, None


def _blocks_product(X: Tensor, Ws: Tensor, perm: Tensor, segs: Tensor, counts: Tensor, sizes) -> Tensor:
    """``Ws (blocks, n_el, C_in, C_out)``; element ``k``'s rows are component-major, so block
    ``b`` of element ``k`` is a contiguous segment of the permuted rows."""
    nb, n_el = Ws.shape[0], Ws.shape[1]
    lead = sum(sizes)
    Y = torch.empty(X.shape[0], Ws.shape[3], dtype=X.dtype, device=X.device)
    packed = pack([Ws[b, k] for b in range(nb) for k in range(n_el)])
    # segment bounds of (element, block) on the device: lead * seg[k] + first component * count
    seg = segs.long() // lead
    cnt = seg[1:] - seg[:-1]
    first = [0]
    for sz in sizes[:-1]:
        first.append(first[-1] + sz)
    bounds = []
    probs = []
    for b, sz in enumerate(sizes):
        lo = segs.long()[:-1] + first[b] * cnt
        hi = lo + sz * cnt
        bounds.append(torch.stack([lo, hi], 1).to(torch.int32))
    bounds = torch.stack(bounds, 0).contiguous()                 # (blocks, n_el, 2)
    for b, sz in enumerate(sizes):
        for k in range(n_el):
            rows = sz * int(counts[k + 1] - counts[k])
            if rows > 0:
                probs.append(MM(X, Ws[b, k], Y, packed[b * n_el + k], perm=perm, seg=bounds[b, k], rows=rows))
    mm(probs)
    return Y


def species_linear_blocks(h: Tensor, z: Tensor, Ws: Sequence[Tensor], sizes: Sequence[int]) -> Tensor:
    """``out[d, i] = h[d, i] @ W_b[z_i]`` for ``h (D, N, C_in)`` whose components ``d`` form blocks
    of ``sizes`` (e.g. ``1, 3, 5, 7`` per degree) and ``Ws[b] (n_el, C_in, C_out)``: every
    (element, block) product in one grouped launch. Float32 CUDA, constant weights."""
    sizes = tuple(int(x) for x in sizes)
    lead = sum(sizes)
    assert h.shape[0] == lead, "h must stack the blocks' components along its first dimension"
    n_el = int(Ws[0].shape[0])
    perm, segs, counts = _grouped_rows(z, n_el, lead)
    X = h.reshape(-1, h.shape[-1])
    X = X if X.is_contiguous() else X.contiguous()
    W = torch.stack([w.detach() for w in Ws], 0).contiguous()
    out = _SpeciesLinearBlocks.apply(X, W, perm, segs, counts, sizes)
    return out.view(*h.shape[:-1], W.shape[-1])


def species_linear(h: Tensor, z: Tensor, Wz: Tensor) -> Tensor:
    """``out[..., i, :] = h[..., i, :] @ Wz[z_i]`` for ``h (..., N, C_in)`` with constant
    ``Wz (n_el, C_in, C_out)``: the rows of every element in one grouped tcgen05 launch (each row
    multiplied by its own element's matrix only). Float32 CUDA; reads the element counts once."""
    n_el, c_in, c_out = Wz.shape
    lead = 1
    for d in h.shape[:-2]:
        lead *= int(d)
    perm, segs, counts = _grouped_rows(z, n_el, lead)
    X = h.reshape(-1, c_in)
    X = X if X.is_contiguous() else X.contiguous()
    out = _SpeciesLinear.apply(X, Wz.detach().contiguous(), perm, segs, counts, lead)
    return out.view(*h.shape[:-1], c_out)
