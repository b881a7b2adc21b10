"""DomainParallel: a structure split over Gloo ranks on the CPU gives the single-process
energy, forces and stress; plans hold, reshard and drive an MD loop."""
import math

import pytest
import torch

from xnn_b200.data import AtomicGraph, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.mace import MACE
from xnn_b200.parallel.domain import DomainParallel, choose_grid

from dist_util import run_ranks

CUT = 3.0


def _model():
    torch.manual_seed(0)
    m = MACE(species=[1, 8], cutoff=CUT, num_channels=8, n_rbf=6, num_interactions=2, max_ell=2,
             correlation=2, avg_num_neighbors=8.0).double()
    return m


def _water(n=162, seed=0):
    s = synthetic.water_box(n, seed=seed)
    return structure_to_graph(s, CUT)


def _molecule(seed=1):
    s = synthetic.organic_molecules(1, seed=seed, labels=False)[0]
    s["atomic_numbers"] = torch.where(s["atomic_numbers"] == 1, 1, 8)
    return structure_to_graph(s, CUT)


def _single(graph, fast):
    m = _model().set_use_fast(fast)
    out = ForceStressOutput(m, compute_stress=graph.cell is not None)(graph.clone())
    return {k: v.detach() for k, v in out.items() if k in ("energy", "forces", "stress")}


def _ranks_eval(rank, world, kind, halo, grid, fast):
    torch.set_default_dtype(torch.float64)
    g = _water() if kind == "water" else _molecule()
    m = _model().set_use_fast(fast)
    dp = DomainParallel(m, halo=halo, grid=grid, skin=0.3)
    out = dp(g)
    plan = dp._plan
    return {"energy": out["energy"], "forces": out["forces"], "stress": out.get("stress"),
            "n_owned": plan.n_owned, "n_ghost": plan.n_ghost, "grid": plan.grid}


def test_choose_grid():
    # cost = prod(1 + 2 halo g / w) over cut axes: (1,2,4) 1.1232 beats (2,2,2) 1.1249
    assert choose_grid(8, [100.0, 100.0, 100.0], 1.0) == (1, 2, 4)
    assert choose_grid(8, [400.0, 100.0, 100.0], 1.0) == (8, 1, 1)
    assert choose_grid(4, [200.0, 20.0, 20.0], 5.0) == (4, 1, 1)
    assert choose_grid(1, [10.0, 10.0, 10.0], 5.0) == (1, 1, 1)


@pytest.mark.parametrize("fast", [False, True])
def test_single_rank_matches_plain(fast):
    torch.set_default_dtype(torch.float64)
    try:
        g = _water()
        ref = _single(g, fast)
        dp = DomainParallel(_model().set_use_fast(fast), skin=0.2)
        out = dp(g)
        torch.testing.assert_close(out["energy"], ref["energy"].reshape(1), rtol=1e-11, atol=1e-10)
        torch.testing.assert_close(out["forces"], ref["forces"], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(out["stress"], ref["stress"], rtol=1e-10, atol=1e-10)
    finally:
        torch.set_default_dtype(torch.float32)


@pytest.mark.parametrize("kind,halo,grid,fast", [
    ("water", "layer", None, False),
    ("water", "field", (2, 1, 1), False),
    ("water", "layer", (1, 2, 1), True),
    ("molecule", "layer", None, False),
])
def test_two_ranks_match_single_process(kind, halo, grid, fast):
    torch.set_default_dtype(torch.float64)
    try:
        g = _water() if kind == "water" else _molecule()
        ref = _single(g, fast)
        outs = run_ranks(_ranks_eval, 2, kind, halo, grid, fast)
    finally:
        torch.set_default_dtype(torch.float32)
    assert sum(o["n_owned"] for o in outs) == g.num_nodes
    assert all(o["n_ghost"] > 0 for o in outs)
    for o in outs:
        torch.testing.assert_close(o["energy"], ref["energy"].reshape(1), rtol=1e-11, atol=1e-10)
        torch.testing.assert_close(o["forces"], ref["forces"], rtol=1e-10, atol=1e-10)
        if kind == "water":
            torch.testing.assert_close(o["stress"], ref["stress"], rtol=1e-10, atol=1e-10)


def _ranks_md(rank, world, steps):
    torch.set_default_dtype(torch.float64)
    from xnn_b200.deploy.md import VelocityVerlet
    g = _water()
    dp = DomainParallel(_model(), skin=0.4)
    md = VelocityVerlet(dp, g, dt_fs=0.5, temperature_k=300.0, seed=3)
    energies = [md.step() for _ in range(steps)]
    pos = md.gather_positions()
    return {"etot": [e["total"] for e in energies], "pos": pos, "rebuilds": md.rebuilds}


def test_md_two_ranks_matches_one():
    torch.set_default_dtype(torch.float64)
    try:
        one = _ranks_md(0, 1, 6)
        two = run_ranks(_ranks_md, 2, 6)
    finally:
        torch.set_default_dtype(torch.float32)
    for o in two:
        torch.testing.assert_close(o["pos"], one["pos"], rtol=1e-9, atol=1e-9)
        assert max(abs(a - b) for a, b in zip(o["etot"], one["etot"])) < 1e-8
