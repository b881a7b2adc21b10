"""Process-group plumbing for one process per GPU (``src/xnn/common/distributed.py``).

``init_process_group`` reads ``RANK / LOCAL_RANK / WORLD_SIZE / MASTER_*`` (torchrun), uses
NCCL for CUDA devices and Gloo on the CPU, binds the rank to ``cuda:LOCAL_RANK`` and
gives the group a bounded timeout so that ranks waiting on a dead peer end with an error.
The helpers sum, gather and shard; every rank must call them in the same order.
"""
from __future__ import annotations

import datetime
import os
from typing import Any, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

DEFAULT_TIMEOUT_S = float(os.environ.get("XNN_PG_TIMEOUT_S", "300"))


def env_world() -> int:
    return int(os.environ.get("WORLD_SIZE", "1"))


def env_rank() -> int:
    return int(os.environ.get("RANK", "0"))


def env_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", "0"))


def is_initialized() -> bool:
    return dist.is_available() and dist.is_initialized()


def world_size() -> int:
    return dist.get_world_size() if is_initialized() else 1


def rank() -> int:
    return dist.get_rank() if is_initialized() else 0


def is_main() -> bool:
    return rank() == 0


def init_process_group(device: Optional[str] = None, timeout_s: Optional[float] = None) -> torch.device:
    """Join the job described by the environment (a no-op for a single process)."""
    want_cuda = (device is None or str(device).startswith("cuda") or device == "auto") and torch.cuda.is_available()
    dev = torch.device(f"cuda:{env_local_rank()}") if want_cuda else torch.device("cpu")
    if want_cuda:
        torch.cuda.set_device(dev)
    if env_world() > 1 and not is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if want_cuda else "gloo"
        kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s or DEFAULT_TIMEOUT_S))
        if want_cuda:
            kw["device_id"] = dev
        dist.init_process_group(**kw)
    return dev


def destroy_process_group() -> None:
    if is_initialized():
        try:
            dist.barrier()
        finally:
            dist.destroy_process_group()


def barrier() -> None:
    if is_initialized():
        dist.barrier()


def shard_indices(n: int, rank_: Optional[int] = None, world: Optional[int] = None) -> List[int]:
    """Strided shard ``rank, rank + world, ...`` of ``range(n)``."""
    r = rank() if rank_ is None else rank_
    w = world_size() if world is None else world
    return list(range(r, n, w))


def all_reduce_sum(t: torch.Tensor) -> torch.Tensor:
    if is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t


def all_reduce_max(t: torch.Tensor) -> torch.Tensor:
    if is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t


def average_gradients(params: Sequence[torch.Tensor]) -> None:
    if not is_initialized():
        return
    w = world_size()
    for p in params:
        if p.grad is not None:
            dist.all_reduce(p.grad, op=dist.ReduceOp.SUM)
            p.grad.div_(w)


def merge_dicts(d: Dict[str, Any]) -> List[Dict[str, Any]]:
    if not is_initialized():
        return [d]
    out: List[Any] = [None] * world_size()
    dist.all_gather_object(out, d)
    return out


def all_gather_cat(t: torch.Tensor) -> torch.Tensor:
    """Rows of every rank concatenated in rank order (padded all-gather of unequal sizes)."""
    if not is_initialized():
        return t
    n = torch.tensor([t.shape[0]], device=t.device, dtype=torch.long)
    sizes = [torch.zeros_like(n) for _ in range(world_size())]
    dist.all_gather(sizes, n)
    m = int(max(s.item() for s in sizes))
    pad = t.new_zeros((m,) + tuple(t.shape[1:]))
    pad[: t.shape[0]] = t
    bufs = [torch.empty_like(pad) for _ in range(world_size())]
    dist.all_gather(bufs, pad)
    return torch.cat([b[: int(s.item())] for b, s in zip(bufs, sizes)])
