"""Data-parallel gradient synchronisation over one flat gradient buffer.

Every trainable parameter's ``.grad`` is a view into one contiguous buffer (the layout
DDP calls "gradient as bucket view"), so the whole reduction is one collective on one
buffer and the backward accumulates straight into it. Two transports:

* ``"nccl"``: ``all_reduce`` (SUM) on the buffer, then a scale by ``1 / world`` -- the
  baseline, and the reference's DDP semantics (``src/xnn/common/train/trainer.py:475-481``);
* ``"p2p"``: :class:`~xnn_b200.parallel.p2p_allreduce.P2PAllReduce`, a single sm_100a
  kernel that reduce-scatters and all-gathers through peer pointers over NVLink and
  fuses the ``1 / world`` scale and the cast (see that module).

Both are plain stream work, so a captured training step records them in its CUDA graph.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from . import distributed as D


class GradSync:
    def __init__(self, params: Sequence[torch.nn.Parameter], backend: str = "auto",
                 dtype: Optional[torch.dtype] = None):
        self.params: List[torch.nn.Parameter] = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        dev = self.params[0].device
        self.dtype = dtype or self.params[0].dtype
        self.numel = sum(p.numel() for p in self.params)
        self.world = D.world_size()
        # pad to a multiple of 64 elements (256-byte aligned slices per rank)
        align = 64 * max(1, self.world)
        self.padded = (self.numel + align - 1) // align * align
        if backend == "auto":
            backend = "nccl"
        if self.world == 1:
            backend = "none"
        self.backend = backend
        self._p2p = None
        if backend == "p2p":
            from .p2p_allreduce import P2PAllReduce
            self._p2p = P2PAllReduce(self.padded, self.dtype, dev)
            self.flat = self._p2p.buffer          # the gradients live in peer-mapped memory
        else:
            self.flat = torch.zeros(self.padded, dtype=self.dtype, device=dev)
        off = 0
        for p in self.params:
            n = p.numel()
            p.grad = self.flat[off:off + n].view_as(p)
            off += n

    def rebind(self) -> None:
        """Point every ``.grad`` at the flat buffer again (after something replaced it)."""
        off = 0
        for p in self.params:
            n = p.numel()
            if p.grad is None or p.grad.data_ptr() != self.flat[off:off + n].data_ptr():
                p.grad = self.flat[off:off + n].view_as(p)
            off += n

    def zero_(self) -> None:
        self.flat.zero_()

    def reduce(self) -> None:
        """Average the gradients over the ranks (in place)."""
        if self.backend == "none":
            return
        if self.backend == "p2p":
            self._p2p.all_reduce_mean_(self.flat)
            return
        dist.all_reduce(self.flat, op=dist.ReduceOp.SUM)
        self.flat.mul_(1.0 / self.world)

    def check(self) -> None:
        """Raise if a fused all-reduce gave up waiting for a peer.

        The kernel reports a timeout in a host-mapped status word, so this read costs no device
        synchronisation; it sees the kernels that have finished by the time it runs. After a
        timeout the ranks hold differently reduced gradients, so training must not go on."""
        if self._p2p is not None:
            self._p2p.check()

    def close(self) -> None:
        if self._p2p is not None:
            self._p2p.close()
            self._p2p = None
