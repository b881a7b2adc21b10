"""Peer-memory buffers and the fused gradient all-reduce kernel (``csrc/p2p_allreduce.cu``).

:class:`PeerBuffer` allocates a device buffer of its own on every rank, exchanges its CUDA IPC
handle over the process group and maps every peer's buffer, so a kernel can load from and
store to any rank's copy over NVLink. :class:`P2PAllReduce` owns one such buffer for the
flat gradients plus a small one for the per-CTA handshake flags, and averages the buffer
over the ranks in one kernel launch (reduce-scatter and all-gather fused, with the
``1 / world`` scale applied once). The kernel's waits are bounded; a timeout is recorded in a
host-mapped status word that :meth:`P2PAllReduce.check` turns into an exception.

``emulate=True`` (tests on one GPU) plays ``world`` ranks inside one cooperative launch over
``world`` local buffers.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from .. import _ext
from . import distributed as D

SPIN_LIMIT = 20_000_000   # polls of ~64 ns: about a second before a wait gives up


class PeerBuffer:
    """A zero-filled device buffer of ``nbytes`` mapped into every rank of the group."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        C = _ext.ops()
        self.device = device
        self.nbytes = int(nbytes)
        self.local, handle = C.ipc_alloc(self.nbytes, device.index)
        self.rank, self.world = D.rank(), D.world_size()
        handles: List[Optional[torch.Tensor]] = [None] * self.world
        if self.world > 1:
            import torch.distributed as dist
            dist.all_gather_object(handles, handle.tolist(), group=group)
        else:
            handles = [handle.tolist()]
        self.ptrs: List[int] = []
        self._opened: List[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.local.data_ptr())
            else:
                p = C.ipc_open(torch.tensor(h, dtype=torch.uint8), device.index)
                self.ptrs.append(p)
                self._opened.append(p)

    def view(self, dtype: torch.dtype, numel: int) -> torch.Tensor:
        return self.local.view(dtype)[:numel]

    def close(self) -> None:
        C = _ext.ops()
        for p in self._opened:
            C.ipc_close(p, self.device.index)
        self._opened = []


class P2PAllReduce:
    def __init__(self, numel: int, dtype: torch.dtype, device: torch.device, nblocks: Optional[int] = None,
                 group=None, emulate_world: int = 0, spin_limit: int = SPIN_LIMIT):
        if dtype != torch.float32:
            raise NotImplementedError("the fused all-reduce reduces float32 gradients")
        C = _ext.ops()
        self.device = device
        self.emulate = emulate_world > 0
        self.world = emulate_world if self.emulate else D.world_size()
        self.rank = 0 if self.emulate else D.rank()
        align = 4 * self.world
        if numel % align:
            raise ValueError(f"numel must be a multiple of {align}")
        self.numel = numel
        flag_bytes = int(C.p2p_flag_words()) * 4
        if self.emulate:
            self._bufs = [PeerBuffer(numel * 4, device) for _ in range(self.world)]
            self._flags = [PeerBuffer(flag_bytes, device) for _ in range(self.world)]
            self.buf_ptrs = [b.ptrs[0] for b in self._bufs]
            self.flag_ptrs = [f.ptrs[0] for f in self._flags]
            self.buffers = [b.view(torch.float32, numel) for b in self._bufs]
            self.buffer = self.buffers[0]
        else:
            self._buf = PeerBuffer(numel * 4, device, group)
            self._flag = PeerBuffer(flag_bytes, device, group)
            self.buf_ptrs = self._buf.ptrs
            self.flag_ptrs = self._flag.ptrs
            self.buffer = self._buf.view(torch.float32, numel)
        self.epochs = torch.zeros(64 * max(1, self.world), dtype=torch.int32, device=device)
        self.status_host, addr = C.mapped_status(1)
        self.status_addr = int(addr.item())
        shard = numel // self.world
        self.nblocks = nblocks or max(1, min(64, (shard + 4095) // 4096))
        self.spin_limit = int(spin_limit)

    def all_reduce_mean_(self, flat: Optional[torch.Tensor] = None, offset: int = 0,
                         numel: Optional[int] = None) -> None:
        """Average ``numel`` elements from ``offset`` of the buffer over the ranks, in place
        (``flat``, when given, must be :attr:`buffer`). A range must be a multiple of
        ``4 * world`` elements long and start on a multiple of 64 elements; every rank reduces
        the same ranges in the same order."""
        if flat is not None and flat.data_ptr() != self.buffer.data_ptr():
            raise ValueError("P2PAllReduce reduces its own peer-mapped buffer")
        n = self.numel - offset if numel is None else int(numel)
        if offset < 0 or n < 0 or offset + n > self.numel or n % (4 * self.world) or offset % 64:
            raise ValueError(f"range [{offset}, {offset + n}) is not a reducible range of {self.numel} elements")
        if n == 0:
            return
        shift = 4 * int(offset)
        nb = self.nblocks if numel is None else max(1, min(self.nblocks, (n // self.world + 4095) // 4096))
        _ext.ops().p2p_allreduce([p + shift for p in self.buf_ptrs], self.flag_ptrs, self.epochs,
                                 self.status_addr, self.world, self.rank, n, 1.0 / self.world, nb,
                                 self.spin_limit, self.emulate)

    def status(self) -> int:
        return int(self.status_host[0].item())

    def check(self) -> None:
        s = self.status()
        if s != 0:
            phase, peer = (s - 100) // 10, (s - 100) % 10
            raise RuntimeError(f"fused all-reduce: rank {self.rank} waited in vain for rank {peer} "
                               f"({'arrival' if phase == 0 else 'departure'}); a peer is late or gone")

    def close(self) -> None:
        if self.emulate:
            for b in self._bufs + self._flags:
                b.close()
        else:
            self._buf.close()
            self._flag.close()
