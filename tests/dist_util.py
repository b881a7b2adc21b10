"""Run a function on ``world`` CPU processes joined by a Gloo process group (127.0.0.1)."""
import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _to_plain(x):
    """Tensors to numpy (pickled by value: no shared-memory handles that die with the child)."""
    import torch
    if isinstance(x, torch.Tensor):
        return ("__tensor__", x.detach().cpu().numpy())
    if isinstance(x, dict):
        return {k: _to_plain(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_to_plain(v) for v in x)
    return x


def _from_plain(x):
    import torch
    if isinstance(x, tuple) and len(x) == 2 and x[0] == "__tensor__":
        return torch.from_numpy(x[1])
    if isinstance(x, dict):
        return {k: _from_plain(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_from_plain(v) for v in x)
    return x


def _entry(rank, world, port, fn, args, queue):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=120))
        out = fn(rank, world, *args)
        queue.put((rank, "ok", _to_plain(out)))
    except Exception:  # pragma: no cover - reported by the parent
        queue.put((rank, "error", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(fn, world: int, *args, timeout: float = 600.0):
    """``fn(rank, world, *args)`` on every rank; returns the results in rank order."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, out = queue.get(timeout=timeout)
            if status != "ok":
                raise RuntimeError(f"rank {rank} failed:\n{out}")
            results[rank] = _from_plain(out)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return [results[r] for r in range(world)]
