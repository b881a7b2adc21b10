"""Ghost-row exchange of :class:`~xnn_b200.parallel.domain.DomainParallel` over peer memory.

One kernel per exchange direction (``csrc/halo_exchange.cu``) packs the rows a rank sends,
stores them directly into the receiving GPUs' buffers over NVLink, waits (bounded) for its own
ghosts to arrive and unpacks them; the adjoint direction returns ghost gradients to the
owners' buffers the same way, and the owners accumulate them into their rows. This replaces
``all_to_all_single`` plus the pack/unpack copies around it (three library calls and two
extra passes over the rows) on the exchange path of a domain-decomposed evaluation.

``emulate_world`` plays several ranks inside one cooperative launch on one GPU (tests).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
from torch import Tensor

from .. import _ext
from . import distributed as D
from .p2p_allreduce import PeerBuffer

MAX_RANKS = 8


def _cumsum(counts: Sequence[int]) -> List[int]:
    out, acc = [], 0
    for c in counts:
        acc += int(c)
        out.append(acc)
    return out


class PeerHaloExchange:
    """Peer buffers, counters and launches of the fused ghost exchange for one device.

    Collective: every rank of the group creates it and calls it in the same order.
    """

    def __init__(self, device: torch.device, group=None, nblocks: int = 64, timeout_s: float = 20.0,
                 emulate_world: int = 0):
        C = _ext.ops()
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.group = group
        self.emulate = emulate_world > 0
        self.world = emulate_world if self.emulate else D.world_size()
        self.rank = 0 if self.emulate else D.rank()
        if not 1 <= self.world <= MAX_RANKS:
            raise ValueError(f"the peer halo exchange supports 1..{MAX_RANKS} ranks, not {self.world}")
        self.nblocks = int(nblocks)
        self.timeout_ns = int(timeout_s * 1e9)
        played = self.world if self.emulate else 1
        if self.emulate:
            self._flags = [PeerBuffer(8 * self.world, self.device) for _ in range(self.world)]
            self.flag_ptrs = [[f.ptrs[0] for f in self._flags]] * played
        else:
            self._flags = [PeerBuffer(8 * self.world, self.device, group)]
            self.flag_ptrs = [list(self._flags[0].ptrs)]
        self.epochs = [torch.zeros(self.nblocks, dtype=torch.int32, device=self.device) for _ in range(played)]
        self.status_host, addr = C.mapped_status(1)
        self.status_addr = int(addr[0])
        self._bufs: List[PeerBuffer] = []
        self.buf_ptrs: List[List[int]] = []
        self.half_bytes = 0

    # ------------------------------------------------------------------ buffers
    def reserve(self, half_bytes: int) -> None:
        """Make each half of every rank's receive buffer at least ``half_bytes``. Collective:
        ``half_bytes`` must be the same on every rank."""
        if half_bytes <= self.half_bytes:
            return
        half = max(int(half_bytes * 1.25), 1 << 20)
        half = (half + 255) // 256 * 256
        if self._bufs:
            torch.cuda.synchronize(self.device)
            if not self.emulate and self.world > 1:
                D.barrier()
            for b in self._bufs:
                b.close()
            if not self.emulate and self.world > 1:
                D.barrier()
        if self.emulate:
            self._bufs = [PeerBuffer(2 * half, self.device) for _ in range(self.world)]
            ptrs = []
            for b in self._bufs:
                ptrs += [b.ptrs[0], b.ptrs[0] + half]
            self.buf_ptrs = [ptrs] * self.world
        else:
            self._bufs = [PeerBuffer(2 * half, self.device, self.group)]
            ptrs = []
            for p in self._bufs[0].ptrs:
                ptrs += [p, p + half]
            self.buf_ptrs = [ptrs]
        self.half_bytes = half

    # ------------------------------------------------------------------ launches
    def launch(self, srcs: List[Tensor], rows: List[Optional[Tensor]], counts: List[Sequence[int]],
               remote_offsets: List[Sequence[int]], outs: List[Tensor], row_bytes: int) -> None:
        """One exchange: rank k sends ``srcs[k][rows[k]]`` (``counts[k][p]`` rows to rank ``p``,
        in rank order) to ``remote_offsets[k][p]`` of rank p's buffer; ``outs[k]`` receives
        rank k's buffer rows."""
        C = _ext.ops()
        C.halo_exchange(srcs, rows, [_cumsum(c) for c in counts], [list(map(int, o)) for o in remote_offsets],
                        outs, self.buf_ptrs, self.flag_ptrs, self.epochs, self.world, self.rank, self.emulate,
                        int(row_bytes), self.status_addr, self.timeout_ns, self.nblocks)

    @staticmethod
    def _row_bytes(x: Tensor) -> int:
        return int(x[0].numel() * x.element_size()) if x.shape[0] else int(
            torch.Size(x.shape[1:]).numel() * x.element_size())

    def forward(self, x: Tensor, plan) -> Tensor:
        """Ghost rows of ``plan`` from their owners' rows ``x`` (``(n_owned, ...)``)."""
        x = x.contiguous()
        rb = self._row_bytes(x)
        self.reserve(plan.max_rows * rb)
        out = x.new_empty((plan.n_ghost,) + tuple(x.shape[1:]))
        self.launch([x], [plan.send_rows], [plan.send_counts], [plan.remote_offsets], [out], rb)
        return out

    def backward(self, g: Tensor, plan, n_owned: int) -> Tensor:
        """Gradient of the owned rows from the ghost rows' gradient ``g`` (``(n_ghost, ...)``)."""
        g = g.contiguous()
        rb = self._row_bytes(g)
        self.reserve(plan.max_rows * rb)
        back = g.new_empty((int(plan.send_rows.shape[0]),) + tuple(g.shape[1:]))
        self.launch([g], [None], [plan.recv_counts], [plan.remote_send_offsets], [back], rb)
        gx = g.new_zeros((n_owned,) + tuple(g.shape[1:]))
        gx.index_add_(0, plan.send_rows, back)
        return gx

    def check(self) -> None:
        """Raise if a wait of an earlier exchange gave up (synchronises the device)."""
        torch.cuda.synchronize(self.device)
        code = int(self.status_host[0])
        if code:
            self.status_host[0] = 0
            raise RuntimeError(f"peer halo exchange: rank {code - 1000} did not arrive in time "
                               f"({self.timeout_ns / 1e9:.1f} s); the exchange results are invalid")

    def close(self) -> None:
        for b in self._bufs + self._flags:
            b.close()
        self._bufs, self._flags = [], []
