"""Data-parallel gradient synchronisation over one flat gradient buffer, bucket by bucket.

Every trainable parameter's ``.grad`` is a view into one contiguous buffer (the layout DDP
calls "gradient as bucket view"). The buffer is cut into *buckets* -- contiguous ranges, each a
group of parameters whose gradients become final together (for the MACE training step: one
interaction block with its product and readout, in the reverse order the backward finishes
them, then everything else). A bucket's reduction can start as soon as the backward has
finished it (:meth:`GradSync.bucket_ready`): it runs on a side stream while the main stream
computes the remaining gradients, and :meth:`GradSync.reduce` launches the buckets not yet
started and makes the main stream wait for all of them before the optimizer reads the
gradients. The reference arms the same overlap through DDP's bucket hooks
(``src/xnn/common/train/trainer.py:475-481``).

Two transports:

* ``"nccl"``: ``all_reduce`` (SUM) of each bucket, then a scale by ``1 / world`` -- the
  baseline, and the reference's DDP semantics;
* ``"p2p"``: :class:`~xnn_b200.parallel.p2p_allreduce.P2PAllReduce`, one sm_100a kernel per
  bucket that reduce-scatters and all-gathers through peer pointers over NVLink with the
  ``1 / world`` scale fused (see that module).

Both are plain stream work, so a captured training step records them (with the side-stream
fork and join) in its CUDA graph.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

from . import distributed as D


class GradSync:
    def __init__(self, params: Sequence[torch.nn.Parameter], backend: str = "auto",
                 dtype: Optional[torch.dtype] = None, buckets: Optional[Sequence[Sequence[torch.nn.Parameter]]] = None):
        self.params: List[torch.nn.Parameter] = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        dev = self.params[0].device
        self.device = dev
        self.dtype = dtype or self.params[0].dtype
        self.world = D.world_size()
        if backend == "auto":
            backend = "nccl"
        if self.world == 1:
            backend = "none"
        self.backend = backend
        # bucket layout: the given groups (trainable members only), then every other parameter
        seen: Dict[int, int] = {}
        groups: List[List[torch.nn.Parameter]] = []
        for grp in (buckets or []):
            keep = [p for p in grp if p.requires_grad and id(p) not in seen and any(p is q for q in self.params)]
            for p in keep:
                seen[id(p)] = len(groups)
            if keep:
                groups.append(keep)
        rest = [p for p in self.params if id(p) not in seen]
        if rest:
            groups.append(rest)
        # each bucket padded to a multiple of 64 * world elements (256-byte aligned slices per rank)
        align = 64 * max(1, self.world)
        self.ranges: List[tuple] = []
        off = 0
        for grp in groups:
            n = sum(p.numel() for p in grp)
            padded = (n + align - 1) // align * align
            self.ranges.append((off, padded))
            off += padded
        self.padded = off
        self.numel = sum(p.numel() for p in self.params)
        self.groups = groups
        self._p2p = None
        if backend == "p2p":
            from .p2p_allreduce import P2PAllReduce
            self._p2p = P2PAllReduce(self.padded, self.dtype, dev)
            self.flat = self._p2p.buffer          # the gradients live in peer-mapped memory
        else:
            self.flat = torch.zeros(self.padded, dtype=self.dtype, device=dev)
        self._slots = []
        for (start, _), grp in zip(self.ranges, groups):
            o = start
            for p in grp:
                n = p.numel()
                self._slots.append((p, o, n))
                p.grad = self.flat[o:o + n].view_as(p)
                o += n
        self.bucket_of = {id(p): i for i, grp in enumerate(groups) for p in grp}
        self._started: List[bool] = [False] * len(groups)
        self._side: Optional[torch.cuda.Stream] = None

    @property
    def n_buckets(self) -> int:
        return len(self.ranges)

    def rebind(self) -> None:
        """Point every ``.grad`` at the flat buffer again (after something replaced it)."""
        for p, o, n in self._slots:
            view = self.flat[o:o + n]
            if p.grad is None or p.grad.data_ptr() != view.data_ptr():
                p.grad = view.view_as(p)

    def zero_(self) -> None:
        self.flat.zero_()
        self._started = [False] * len(self.ranges)

    # ------------------------------------------------------------------ reduction
    def _side_stream(self) -> torch.cuda.Stream:
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.device)
        return self._side

    def _launch(self, i: int) -> None:
        start, n = self.ranges[i]
        view = self.flat[start:start + n]
        if self.device.type != "cuda":
            dist.all_reduce(view, op=dist.ReduceOp.SUM)
            view.mul_(1.0 / self.world)
        else:
            # forked from the current stream, so the bucket's reduction follows the work that
            # produced it and overlaps what the current stream does next
            side = self._side_stream()
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                if self.backend == "p2p":
                    self._p2p.all_reduce_mean_(offset=start, numel=n)
                else:
                    dist.all_reduce(view, op=dist.ReduceOp.SUM)
                    view.mul_(1.0 / self.world)
        self._started[i] = True

    def bucket_ready(self, i: int) -> None:
        """Bucket ``i``'s gradients are final: start its reduction (overlapping what follows)."""
        if self.backend == "none" or self._started[i]:
            return
        self._launch(i)

    def reduce(self) -> None:
        """Average the gradients over the ranks (in place): starts the buckets not yet started
        and joins every reduction into the current stream."""
        if self.backend == "none":
            return
        for i, started in enumerate(self._started):
            if not started:
                self._launch(i)
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).wait_stream(self._side_stream())

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
