"""Index reductions shared by every model, and the domain-decomposition hooks.

``scatter_sum`` / ``gather_rows`` / ``structure_sum`` keep the reference's semantics
(``src/xnn/common/models/ops.py:403,494,531``): per-structure energies are summed in
float64. ``refresh_ghosts`` and ``whole_structure_sum`` are identity / plain sums
outside a :class:`~xnn_b200.parallel.domain.DomainParallel` evaluation; inside one the
active plan (a thread-local) exchanges ghost rows and sums over ranks
(``ops.py:576-645``).
"""
from __future__ import annotations

import threading
from typing import Optional

import torch
from torch import Tensor

_DOMAIN = threading.local()


def scatter_sum(src: Tensor, index: Tensor, dim_size: int, dim: int = 0) -> Tensor:
    """``out[index[e]] += src[e]`` along ``dim`` (``out`` has ``dim_size`` rows)."""
    shape = list(src.shape)
    shape[dim] = dim_size
    out = src.new_zeros(shape)
    return out.index_add(dim, index, src)


def gather_rows(x: Tensor, index: Tensor) -> Tensor:
    return x.index_select(0, index)


def structure_sum(values: Tensor, batch: Tensor, num_graphs: int) -> Tensor:
    """Per-structure sums in float64 (``values`` is per atom, ``(N, ...)``)."""
    v = values.to(torch.float64)
    out = v.new_zeros((num_graphs,) + tuple(v.shape[1:]))
    return out.index_add(0, batch, v)


def segment_softmax(logits: Tensor, index: Tensor, n: int, weight: Optional[Tensor] = None) -> Tensor:
    """Softmax of ``logits`` within the groups given by ``index`` (``n`` groups). With a per-row
    ``weight`` ``u`` (a cutoff envelope): ``u_r e^{z_r} / (1 + sum_s u_s e^{z_s})`` -- a null key of
    logit zero lets the last row of a group fade out continuously (the Equiformers' smooth form)."""
    shape = (n,) + tuple(logits.shape[1:])
    idx = index.view((-1,) + (1,) * (logits.dim() - 1)).expand_as(logits)
    mx = logits.new_full(shape, float("-inf")).scatter_reduce(0, idx, logits.detach(), "amax", include_self=True)
    if weight is None:
        e = torch.exp(logits - mx.index_select(0, index))
        return e / (scatter_sum(e, index, n) + 1e-16).index_select(0, index)
    mx = mx.clamp(min=0.0)
    e = torch.exp(logits - mx.index_select(0, index)) * weight.view((-1,) + (1,) * (logits.dim() - 1))
    return e / (scatter_sum(e, index, n) + torch.exp(-mx)).index_select(0, index)


def cell_volume(cell: Tensor) -> Tensor:
    """``|a . (b x c)|`` per cell (``(B, 3, 3)`` -> ``(B,)``)."""
    return torch.linalg.det(cell).abs()


def build_triplets(edge_index: Tensor, n_nodes: int):
    """All ordered pairs of distinct edges sharing a receiver: ``(edge_ji, edge_ki)`` index pairs."""
    dst = edge_index[1]
    order = torch.argsort(dst, stable=True)
    counts = torch.bincount(dst, minlength=n_nodes)
    starts = torch.cumsum(counts, 0) - counts
    deg = counts[dst[order]]
    reps = deg
    e1 = torch.repeat_interleave(order, reps)
    local = torch.arange(e1.numel(), device=dst.device) - torch.repeat_interleave(
        torch.cumsum(reps, 0) - reps, reps)
    e2 = order[starts[dst[e1]] + local]
    keep = e1 != e2
    return e1[keep], e2[keep]


def build_center_pairs(dst: Tensor, n_nodes: int):
    """All unordered pairs of distinct edges sharing a receiver, as ``(first, second)`` edge
    indices with ``first`` before ``second`` in the receiver's (stable) edge order."""
    order = torch.argsort(dst, stable=True)
    counts = torch.bincount(dst, minlength=n_nodes)
    starts = torch.cumsum(counts, 0) - counts
    d = dst.index_select(0, order)
    local = torch.arange(order.numel(), device=dst.device) - starts.index_select(0, d)
    partners = counts.index_select(0, d) - 1 - local               # later edges of the same receiver
    first = torch.repeat_interleave(order, partners)
    base = torch.repeat_interleave(torch.arange(order.numel(), device=dst.device), partners)
    k = torch.arange(first.numel(), device=dst.device) - torch.repeat_interleave(
        torch.cumsum(partners, 0) - partners, partners)
    second = order.index_select(0, base + 1 + k)
    return first, second


# --- domain-decomposition hooks --------------------------------------------------------
def active_domain():
    return getattr(_DOMAIN, "plan", None)


def refresh_ghosts(x: Tensor) -> Tensor:
    """Ghost rows of ``x`` replaced by their owners' values (identity outside a domain evaluation)."""
    plan = active_domain()
    if plan is None:
        return x
    return plan.refresh(x)


def whole_structure_sum(values: Tensor, batch: Tensor, num_graphs: int) -> Tensor:
    """A per-structure sum over all ranks' owned atoms (plain sum outside a domain evaluation)."""
    plan = active_domain()
    if plan is None:
        return structure_sum(values, batch, num_graphs)
    return plan.whole_sum(values, batch, num_graphs)


class domain_hooks:
    """Context manager installing ``plan`` as the active domain of this thread."""

    def __init__(self, plan: Optional[object]):
        self.plan = plan
        self.prev = None

    def __enter__(self):
        self.prev = getattr(_DOMAIN, "plan", None)
        _DOMAIN.plan = self.plan
        return self.plan

    def __exit__(self, *exc):
        _DOMAIN.plan = self.prev
        return False
