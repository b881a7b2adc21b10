"""Failure detection without a GPU fault: failures are made on the host.

* a fused all-reduce that reports a timeout in its status word (a fake of the failing kernel's
  report, read through the real check) stops training with an error naming the peer;
* a rank that leaves between steps makes the next collective of the remaining rank raise
  instead of hanging (two Gloo ranks on the CPU).
"""
import os

import pytest
import torch

from dist_util import run_ranks
from xnn_b200.data import synthetic


def _cfg(tmp_path, extra=None):
    from xnn_b200.config import from_dict
    d = {
        "model": {"name": "schnet", "cutoff": 4.0, "n_features": 8, "n_interactions": 1, "n_rbf": 6},
        "optim": {"lr": 1e-3, "epochs": 1, "force_weight": 1.0, "scheduler": "none"},
        "data": {"batch_size": 2, "val_fraction": 0.0},
        "trainer": {"loggers": [], "cuda_graph": False},
        "device": "cpu", "seed": 3, "output_dir": str(tmp_path),
    }
    if extra:
        d.update(extra)
    return from_dict(d)


def _data(n, seed):
    from xnn_b200.data import AtomicDataset
    return AtomicDataset(synthetic.small_organic(n, seed=seed), 4.0)


class _TimedOutAllReduce:
    """Stands in for :class:`~xnn_b200.parallel.p2p_allreduce.P2PAllReduce` after its kernel gave
    up waiting for rank 1 at the arrival handshake (status code 100 + phase * 10 + peer)."""

    def __init__(self):
        from xnn_b200.parallel.p2p_allreduce import P2PAllReduce
        self._real = object.__new__(P2PAllReduce)
        self._real.rank = 0
        self._real.status_host = torch.tensor([101], dtype=torch.int32)

    def check(self):
        self._real.check()

    def close(self):
        pass


def test_fused_allreduce_timeout_stops_training(tmp_path):
    from xnn_b200.train import Trainer
    tr = Trainer(_cfg(tmp_path), _data(4, 1))
    batch = next(iter(tr._loader(tr.train_set, train=True)))
    tr.train_step(batch)                       # healthy step
    tr.grad_sync._p2p = _TimedOutAllReduce()   # the next kernel report says: rank 1 never arrived
    with pytest.raises(RuntimeError, match="waited in vain for rank 1"):
        tr.train_step(batch)


def _leaving_rank(rank, world, out_dir):
    import torch.distributed as dist

    from xnn_b200.train import Trainer
    tr = Trainer(_cfg(out_dir), _data(8, 5))
    batch = next(iter(tr._loader(tr.train_set, train=True)))
    tr.train_step(batch)
    dist.barrier()
    if rank == 1:
        return "left"                          # leaves between steps, with nothing in flight
    try:
        for _ in range(5):
            tr.train_step(batch)               # the gradient all-reduce needs rank 1
    except Exception as exc:                   # noqa: BLE001 - any error, as long as it is not a hang
        return f"raised: {type(exc).__name__}"
    return "no error"


def test_rank_that_leaves_between_steps_makes_the_next_collective_raise(tmp_path):
    out = run_ranks(_leaving_rank, 2, str(tmp_path), timeout=300)
    assert out[1] == "left"
    assert out[0].startswith("raised"), out[0]


def _corrupt_plan(rank, world):
    from xnn_b200.data import structure_to_graph
    from xnn_b200.models.mace import MACE
    from xnn_b200.parallel import domain
    torch.set_default_dtype(torch.float64)
    if rank == 1:
        real = domain._ghost_counts
        domain._ghost_counts = lambda owner, w: real(owner, w) + torch.nn.functional.one_hot(  # noqa: E731
            torch.tensor(0), w).to(owner.device)                     # one ghost too many from rank 0
    torch.manual_seed(0)
    m = MACE(species=[1, 8], cutoff=3.0, num_channels=8, n_rbf=6, num_interactions=2, max_ell=2,
             correlation=2, avg_num_neighbors=8.0).double()
    g = structure_to_graph(synthetic.water_box(162, seed=0), 3.0)
    dp = domain.DomainParallel(m, skin=0.3)
    try:
        dp.plan(g)
    except domain.PlanError as exc:
        return f"raised: {exc}"
    return "no error"


def test_corrupted_ghost_count_makes_every_rank_raise():
    out = run_ranks(_corrupt_plan, 2, timeout=300)
    assert all(o.startswith("raised") for o in out), out
