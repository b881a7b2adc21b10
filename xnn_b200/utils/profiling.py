"""Tracing helpers: named regions and per-kernel time tables.

* :func:`region` names a stretch of host code. Under ``torch.profiler`` it appears as a
  ``record_function`` range, and with ``XNN_B200_NVTX=1`` (or inside
  ``torch.autograd.profiler.emit_nvtx``) it also pushes an NVTX range for external
  timeline tools. Outside both it costs one dictionary lookup. The reference wraps its PME and
  induction stages the same way (``src/xnn/ffnn/models/amoeba_ewald.py:67-80``).
* :func:`kernel_table` runs a callable under ``torch.profiler`` and returns every GPU kernel it
  launched with its count and summed device time, plus the share of device time and launches
  that belong to this package's own kernels (those compiled into ``xnn_b200/_C.so``).

``python -m xnn_b200.utils.profiling [--model tensornet|pme]`` prints that table for one eager
training step of the benchmark configuration (MACE: 64 organic molecules, 96 channels;
TensorNet: 32 crystals, 64 channels, energy + force + stress loss) or one evaluation of the
polarizable-multipole PME workload (``--batch`` atoms, 100,000 by default) or one step of the
domain-decomposed MD of a water box (``--model md``, ``--batch`` atoms, 1,000,000 by default).
"""
from __future__ import annotations

import argparse
import contextlib
import functools
import os
import re
from collections import defaultdict
from pathlib import Path
from typing import Callable, Dict, List

import torch

_NVTX = os.environ.get("XNN_B200_NVTX", "0") == "1"

_GLOBAL = re.compile(r"__global__\s+(?:__launch_bounds__\s*\([^)]*\)\s*)?(?:static\s+)?void\s+"
                     r"(?:__launch_bounds__\s*\([^)]*\)\s*)?(\w+)\s*\(")


@functools.lru_cache(maxsize=1)
def own_kernel_names() -> frozenset:
    """Names of the ``__global__`` functions in this package's CUDA sources (``csrc``)."""
    root = Path(__file__).resolve().parents[1] / "csrc"
    names = set()
    for f in sorted(root.rglob("*")):
        if f.suffix in (".cu", ".cuh", ".h"):
            names.update(_GLOBAL.findall(f.read_text(errors="replace")))
    return frozenset(names)


def kernel_base_name(name: str) -> str:
    """``void (anonymous namespace)::gemm_ws_kernel<32>(CUtensorMap_st, ...)`` -> ``gemm_ws_kernel``."""
    out, level = [], 0
    for ch in name:                       # drop template arguments (they may hold parentheses)
        if ch == "<":
            level += 1
        elif ch == ">":
            level -= 1
        elif level == 0:
            out.append(ch)
    flat = "".join(out).replace("(anonymous namespace)::", "").split("(", 1)[0].strip()
    return flat.split()[-1].split("::")[-1] if flat else ""


def is_own_kernel(name: str) -> bool:
    """Whether a profiler kernel name is one of this package's kernels."""
    return kernel_base_name(name) in own_kernel_names()


@contextlib.contextmanager
def region(name: str):
    """A named range for profilers (record_function; NVTX when enabled)."""
    nvtx = _NVTX and torch.cuda.is_available()
    if nvtx:
        torch.cuda.nvtx.range_push(name)
    try:
        with torch.profiler.record_function(name):
            yield
    finally:
        if nvtx:
            torch.cuda.nvtx.range_pop()


def kernel_table(fn: Callable[[], object], warmup: int = 1, ops: bool = False,
                 stacks: int = 0) -> Dict[str, object]:
    """GPU kernels launched by one call of ``fn`` (after ``warmup`` untimed calls); with ``ops``
    also the host operators that launched device work, by count (``"ops"``); with ``stacks`` the
    Python call sites (``stacks`` frames deep) of the host operators with the most device time."""
    from torch.profiler import ProfilerActivity, profile
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    acts = [ProfilerActivity.CUDA] + ([ProfilerActivity.CPU] if (ops or stacks) else [])
    with profile(activities=acts, with_stack=bool(stacks)) as prof:
        fn()
        torch.cuda.synchronize()
    count: Dict[str, int] = defaultdict(int)
    us: Dict[str, float] = defaultdict(float)
    for e in prof.events():
        if e.device_type.name != "CUDA" or getattr(e, "is_user_annotation", False):
            continue                    # a record_function range spans kernels counted on their own
        count[e.name] += 1
        us[e.name] += float(getattr(e, "device_time", 0.0) or getattr(e, "cuda_time", 0.0) or 0.0)
    rows: List[Dict[str, object]] = [
        {"kernel": k, "launches": count[k], "us": round(us[k], 2), "own": is_own_kernel(k)} for k in count]
    rows.sort(key=lambda r: -float(r["us"]))
    tot_us = sum(float(r["us"]) for r in rows)
    own_us = sum(float(r["us"]) for r in rows if r["own"])
    tot_n = sum(int(r["launches"]) for r in rows)
    own_n = sum(int(r["launches"]) for r in rows if r["own"])
    out = {"rows": rows, "device_us": round(tot_us, 1), "launches": tot_n, "own_launches": own_n,
           "own_time_share": round(own_us / tot_us, 4) if tot_us else None}
    if ops:
        avg = [k for k in prof.key_averages() if getattr(k, "self_device_time_total", 0) > 0]
        avg.sort(key=lambda k: -k.count)
        out["ops"] = [{"op": k.key, "calls": k.count, "us": round(float(k.self_device_time_total), 1)} for k in avg]
    if stacks:
        avg = [k for k in prof.key_averages(group_by_stack_n=stacks)
               if getattr(k, "self_device_time_total", 0) > 0 and k.key.startswith("aten::")]
        avg.sort(key=lambda k: -float(k.self_device_time_total))
        out["sites"] = [{"op": k.key, "calls": k.count, "us": round(float(k.self_device_time_total), 1),
                         "stack": [f for f in (k.stack or []) if "torch/" not in f][:stacks]} for k in avg]
    return out


def _mace_step(batch: int):
    import tempfile

    from ..config import from_dict
    from ..data import AtomicDataset, synthetic
    from ..train import Trainer
    mols = synthetic.organic_molecules(batch, seed=1000)
    ds = AtomicDataset(mols, 4.5, precompute=True)
    graphs = [ds[i] for i in range(len(ds))]
    avg = sum(g.num_edges for g in graphs) / sum(g.num_nodes for g in graphs)
    cfg = from_dict({
        "model": {"name": "mace", "cutoff": 4.5, "n_features": 96, "n_interactions": 2, "n_rbf": 8,
                  "extra": {"species": [1, 6, 7, 8, 9, 16, 17], "max_ell": 3, "max_L": 0, "correlation": 3,
                            "avg_num_neighbors": avg}},
        "optim": {"lr": 1e-3, "energy_weight": 1.0, "force_weight": 10.0, "epochs": 1, "scheduler": "none"},
        "data": {"batch_size": batch, "val_fraction": 0.0},
        "trainer": {"cuda_graph": False, "loggers": []},
        "device": "cuda", "seed": 1234, "output_dir": tempfile.mkdtemp(prefix="xnn_b200_prof_"),
    })
    tr = Trainer(cfg, ds, val=[], test=[])
    cap = tr.capacity_for_batches([graphs])
    b = tr.make_padder(*cap)(graphs).to(tr.device)
    return lambda: tr._train_step_impl(b)


def _tensornet_step(batch: int):
    import tempfile

    from ..config import from_dict
    from ..data import AtomicDataset, collate, synthetic
    from ..train import Trainer
    structs = synthetic.triclinic_crystals(batch, seed=3000)
    ds = AtomicDataset(structs, 5.0, precompute=True)
    cfg = from_dict({
        "model": {"name": "tensornet", "cutoff": 5.0, "n_features": 64, "n_interactions": 2, "n_rbf": 32,
                  "extra": {"n_elements": 90}},
        "optim": {"lr": 1e-3, "energy_weight": 1.0, "force_weight": 10.0, "stress_weight": 1.0, "epochs": 1,
                  "scheduler": "none"},
        "data": {"batch_size": batch, "val_fraction": 0.0},
        "trainer": {"cuda_graph": False, "loggers": []},
        "device": "cuda", "seed": 1234, "output_dir": tempfile.mkdtemp(prefix="xnn_b200_prof_"),
    })
    tr = Trainer(cfg, ds, val=[], test=[])
    b = collate([ds[i] for i in range(len(ds))]).to(tr.device)
    return lambda: tr.train_step(b)


def _pme_eval(atoms: int):
    from ..ffnn import multipoles as MP
    from ..ffnn.water import multipole_water
    dev = torch.device("cuda", torch.cuda.current_device())
    w = multipole_water(atoms, seed=0, device=dev)
    setup = MP.EwaldSetup(alpha=0.4, cutoff=7.0, mesh=(128, 128, 128), order=5, fft_dtype=torch.float32)
    mod = MP.PolarizableMultipoles(setup, tol_debye=1e-5, max_iter=100)
    return lambda: mod(w["pos"], w["cell"], w["q"], w["d"], w["Q"], w["pol"], w["molecule"])


def _md_step(atoms: int, chunk: int = 4_000_000):
    from ..data import synthetic
    from ..data.atomic_graph import AtomicGraph
    from ..deploy.md import VelocityVerlet
    from ..models.mace import MACE
    from ..parallel.domain import DomainParallel
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(4321)
    model = MACE(species=[1, 6, 7, 8, 9, 16, 17], cutoff=4.5, num_channels=96, n_rbf=8, num_interactions=2,
                 max_ell=3, correlation=3, avg_num_neighbors=38.0).to(dev).eval()
    model.edge_chunk = chunk
    s = synthetic.water_box(atoms, seed=0)
    n = int(s["pos"].shape[0])
    g = AtomicGraph(pos=s["pos"].to(dev), atomic_numbers=s["atomic_numbers"].to(dev),
                    edge_index=torch.zeros(2, 0, dtype=torch.long, device=dev),
                    cell_shifts=torch.zeros(0, 3, dtype=torch.long, device=dev),
                    batch=torch.zeros(n, dtype=torch.long, device=dev), n_atoms=torch.tensor([n], device=dev),
                    cell=s["cell"][None].to(dev), pbc=s["pbc"][None].to(dev))
    md = VelocityVerlet(DomainParallel(model, skin=1.0), g, dt_fs=0.5, temperature_k=300.0, seed=7)
    return lambda: md.step()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="mace", choices=["mace", "tensornet", "pme", "md"])
    ap.add_argument("--batch", type=int, default=None, help="structures per step (64 MACE, 32 TensorNet)")
    ap.add_argument("--top", type=int, default=40)
    ap.add_argument("--json", default=None, help="also write the table as JSON to this path")
    ap.add_argument("--ops", action="store_true", help="also list the host operators that launched device work")
    ap.add_argument("--stacks", type=int, default=0, help="also list the call sites (this many frames) of the "
                                                          "ATen operators with the most device time")
    a = ap.parse_args(argv)
    if a.model == "mace":
        fn = _mace_step(a.batch or 64)
    elif a.model == "tensornet":
        fn = _tensornet_step(a.batch or 32)
    elif a.model == "pme":
        fn = _pme_eval(a.batch or 100_000)
    else:
        fn = _md_step(a.batch or 1_000_000)
    tab = kernel_table(fn, warmup=3, ops=a.ops, stacks=a.stacks)
    print(f"launches {tab['launches']} (own {tab['own_launches']}), device time {tab['device_us']} us, "
          f"own-kernel share {tab['own_time_share']}")
    for r in tab["rows"][:a.top]:
        print(f"{r['us']:10.1f} us {r['launches']:5d}  {'*' if r['own'] else ' '} {r['kernel'][:120]}")
    if a.ops:
        print("host operators launching device work (calls, device us):")
        for r in tab["ops"][:a.top]:
            print(f"{r['calls']:6d} {r['us']:10.1f} us  {r['op'][:100]}")
    if a.stacks:
        print("ATen call sites by device time (calls, device us, frames):")
        for r in tab["sites"][:a.top]:
            print(f"{r['calls']:6d} {r['us']:10.1f} us  {r['op']}  <- " + " <- ".join(r["stack"]))
    if a.json:
        import json
        with open(a.json, "w") as f:
            json.dump(tab, f, indent=1)


if __name__ == "__main__":
    main()
