"""Gradient all-reduce microbenchmark: the fused peer-memory kernel against NCCL.

Run one process per GPU::

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m xnn_b200.benchmark.collectives --sizes-mb 1.6 16 64 256

Every size is averaged (``1 / world`` scale included) in place, timed with CUDA events on the
launching stream after warm-up, the maximum over ranks reported. The NVLink roofline of an
average of ``S`` bytes over ``W`` GPUs: a reduce-scatter plus an all-gather moves
``2 (W - 1) / W * S`` bytes out of (and into) every GPU, so the lower bound on the time is those
bytes over the per-direction link bandwidth (770 GB/s measured for a peer copy on this class of
machine; 900 GB/s nominal). ``frac_of_link`` is that bound over the measured time.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes-mb", type=float, nargs="+", default=[1.6, 16.0, 64.0, 256.0])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()
    from datetime import timedelta
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", local))
    from xnn_b200.parallel.p2p_allreduce import P2PAllReduce
    W, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", local)
    rows = []
    for mb in args.sizes_mb:
        n = int(mb * 2 ** 20 / 4)
        n = (n + 64 * W - 1) // (64 * W) * (64 * W)
        ar = P2PAllReduce(n, torch.float32, dev)
        ar.buffer.normal_()
        nccl_buf = torch.randn(n, device=dev)

        def nccl():
            dist.all_reduce(nccl_buf)
            nccl_buf.mul_(1.0 / W)

        t_p2p = _time(ar.all_reduce_mean_, args.iters, args.warmup)
        ar.check()
        t_nccl = _time(nccl, args.iters, args.warmup)
        S = 4 * n
        wire = 2 * (W - 1) / W * S
        bound_ms = wire / (LINK_GBS * 1e9) * 1e3
        rows.append({"mb": round(S / 2 ** 20, 2), "p2p_ms": round(t_p2p, 4), "nccl_ms": round(t_nccl, 4),
                     "p2p_busbw_gbs": round(wire / t_p2p / 1e6, 1), "nccl_busbw_gbs": round(wire / t_nccl / 1e6, 1),
                     "frac_of_link_p2p": round(bound_ms / t_p2p, 3), "frac_of_link_nccl": round(bound_ms / t_nccl, 3),
                     "p2p_ctas": ar.nblocks})
        ar.close()
    if rank == 0:
        print(json.dumps({"bench": "gradient all-reduce (mean, fp32, in place)", "world": W,
                          "link_gbs_per_direction": LINK_GBS, "rows": rows}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
