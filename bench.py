"""Headline benchmark: MACE (OFF23-small-shaped) data-parallel training throughput, structures/s.

Config 2 of the benchmark plan: MACE with 2 interactions, 96x0e hidden channels, max_L 0,
correlation 3, max_ell 3, 8 Bessel functions, r_max 4.5 A, float32, random init; per GPU a
batch of 64 seeded synthetic molecules of 10-60 atoms ({H,C,N,O,F,S,Cl} at 50/30/8/8/2/1/1 %,
0.1 atoms/A^3, 0.9 A minimum separation) with float64 Morse labels; energy + force loss.
One process per GPU (torchrun), NCCL; weak scaling (64 structures per GPU per step).

Device timing: W untimed warm-up steps, then K steps each bracketed by CUDA events on the
launching stream, with a 256 MB write (larger than the 126 MB L2) between steps to flush
L2; barrier + synchronize on both sides; the max over ranks is reported. The e2e figure runs
the same steps through ``Trainer.train_step`` on batches in pinned host memory (host-to-device
copy of every step's inputs) and reads each step's loss back to the host.

``--impl reference`` runs the reference package installed under ``baseline/_ref`` through
its own API, or prints why it cannot.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))


# name fragments of the kernels compiled into xnn_b200/_C.so
OUR_KERNELS = ("conv_gather", "conv_edge", "conv_scatter", "symcon_", "edge_geom_", "p2p_allreduce", "halo_exchange",
               "gemm_pack_kernel", "gemm_rows_kernel", "gemm_reduce_kernel", "gemm_ws_kernel", "gemm_ws_pack_kernel",
               "gemm_reduce_ws_kernel", "sum_partials_kernel", "radial_basis_kernel", "radial_act_kernel",
               "radial_dact_kernel", "nb_count", "nb_write", "mp_real_kernel", "pme_spread_kernel",
               "pme_gather_kernel", "node_mm_kernel", "node_mmT_kernel", "node_sum_kernel", "node_pack",
               "species_sort_kernel")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="xnn_b200", choices=["xnn_b200", "reference"])
    ap.add_argument("--batch", type=int, default=64, help="structures per GPU per step")
    ap.add_argument("--pool", type=int, default=8, help="distinct batches per rank, cycled")
    ap.add_argument("--no-graph", action="store_true", help="eager steps instead of one CUDA graph")
    ap.add_argument("--grad-sync", default="nccl", choices=["nccl", "p2p"])
    ap.add_argument("--dtype", default="float32")
    ap.add_argument("--md-atoms", type=int, default=1_000_000, help="atoms of the MD water box (0: skip MD)")
    ap.add_argument("--md-steps", type=int, default=10)
    ap.add_argument("--md-warmup", type=int, default=3)
    ap.add_argument("--md-exchange", default="p2p", choices=["collective", "p2p"])
    ap.add_argument("--md-chunk", type=int, default=4_000_000, help="edges per chunk of the lean force pass")
    ap.add_argument("--pme-atoms", type=int, default=100_000, help="atoms of the config-5 water box (0: skip)")
    ap.add_argument("--pme-steps", type=int, default=3)
    ap.add_argument("--pme-exchange", default="collective", choices=["collective", "p2p"])
    return ap.parse_args()


def pme_measure(args, dev, world, rank):
    """Config 5: polarizable multipoles with PME (128^3, order 5, alpha 0.4, 7 A real space, CG
    induction to 1e-5 D), energy and forces per evaluation; the mesh z-slab decomposed over the
    ranks (distributed 3D FFT), real-space pairs split, fields / forces summed."""
    import torch
    import torch.distributed as dist

    from xnn_b200.ffnn import multipoles as MP
    from xnn_b200.ffnn.slab_fft import SlabFFT
    from xnn_b200.ffnn.water import multipole_water

    w = multipole_water(args.pme_atoms, seed=0, device=dev)
    setup = MP.EwaldSetup(alpha=0.4, cutoff=7.0, mesh=(128, 128, 128), order=5, fft_dtype=torch.float32)
    backend = SlabFFT(list(setup.mesh), exchange=args.pme_exchange) if world > 1 else None
    mod = MP.PolarizableMultipoles(setup, tol_debye=1e-5, max_iter=100, mesh_backend=backend)
    run = lambda: mod(w["pos"], w["cell"], w["q"], w["d"], w["Q"], w["pol"], w["molecule"])  # noqa: E731
    out = run()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    for _ in range(args.pme_steps):
        out = run()
        e = float(out["energy"])
    b.record()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    t = torch.tensor([a.elapsed_time(b) / args.pme_steps, wall / args.pme_steps * 1e3], device=dev,
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, wall_ms = float(t[0]), float(t[1])
    if backend is not None:
        backend.close()
    return {"metric": "AMOEBA-style PME evaluations/s", "value": round(1e3 / ms, 3), "unit": "evaluations/s",
            "ms_per_step": round(ms, 2), "steps": args.pme_steps, "warmup": 1, "atoms": int(w["pos"].shape[0]),
            "cg_iterations": int(out["iterations"]), "residual_debye": float(out["residual_debye"]),
            "energy_ev": e,
            "config": {"mesh": [128, 128, 128], "order": 5, "alpha": 0.4, "cutoff_A": 7.0, "tol_debye": 1e-5,
                       "real_space": "float64", "fft": "float32", "decomposition": f"z-slab x{world}",
                       "exchange": args.pme_exchange if world > 1 else "none",
                       "box": "water density (0.1 atoms/A^3): 100.4 A for 100,000 atoms"},
            "e2e": {"value": round(1e3 / wall_ms, 3), "unit": "evaluations/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 8}}


def md_measure(args, dev, world, rank):
    """Config-4 MD: velocity Verlet on a periodic water box, domain-decomposed over the ranks.

    Returns the JSON fragment (atom-steps/s over all ranks, device-timed, max over ranks)."""
    import torch
    import torch.distributed as dist

    from xnn_b200.data import synthetic
    from xnn_b200.data.atomic_graph import AtomicGraph
    from xnn_b200.deploy.md import VelocityVerlet
    from xnn_b200.models.mace import MACE
    from xnn_b200.parallel.domain import DomainParallel

    torch.manual_seed(4321)
    model = MACE(species=[1, 6, 7, 8, 9, 16, 17], cutoff=4.5, num_channels=96, n_rbf=8, num_interactions=2,
                 max_ell=3, correlation=3, avg_num_neighbors=38.0).to(dev).eval()
    model.edge_chunk = args.md_chunk
    s = synthetic.water_box(args.md_atoms, seed=0)
    N = int(s["pos"].shape[0])
    g = AtomicGraph(pos=s["pos"].to(dev), atomic_numbers=s["atomic_numbers"].to(dev),
                    edge_index=torch.zeros(2, 0, dtype=torch.long, device=dev),
                    cell_shifts=torch.zeros(0, 3, dtype=torch.long, device=dev),
                    batch=torch.zeros(N, dtype=torch.long, device=dev), n_atoms=torch.tensor([N], device=dev),
                    cell=s["cell"][None].to(dev), pbc=s["pbc"][None].to(dev))
    dp = DomainParallel(model, skin=1.0, exchange=args.md_exchange if world > 1 else "collective")
    md = VelocityVerlet(dp, g, dt_fs=0.5, temperature_k=300.0, seed=7)
    del g, s
    for _ in range(max(3, args.md_warmup)):
        md.step()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.md_steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.md_steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    log = None
    for i in range(args.md_steps):
        starts[i].record()
        log = md.step()
        stops[i].record()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    if world > 1:
        dist.barrier()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, stops)) / args.md_steps
    t = torch.tensor([ms, wall], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, wall_max = float(t[0]), float(t[1])
    out = {"metric": "1M-atom MD atom-steps/s" if N >= 999_999 else f"{N}-atom MD atom-steps/s",
           "value": round(N / (ms_max / 1e3), 1), "unit": "atom-steps/s", "ms_per_step": round(ms_max, 3),
           "steps": args.md_steps, "warmup": max(3, args.md_warmup), "atoms": N,
           "config": {"model": "config-2 MACE, random init", "box": "periodic water, 0.1 atoms/A^3",
                      "integrator": "velocity Verlet, dt 0.5 fs, 300 K start", "grid": list(md.plan.grid),
                      "halo": dp.halo, "skin_A": 1.0, "exchange": dp.exchange if world > 1 else "none",
                      "edge_chunk": args.md_chunk, "rebuilds_in_run": md.rebuilds,
                      "l2": "per-step working set (GBs) far larger than L2"},
           "e2e": {"value": round(N * args.md_steps / wall_max, 1), "unit": "atom-steps/s",
                   "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 16,
                   "note": "wall clock of VelocityVerlet.step(), which reads back the energies every step"},
           "energy_total_ev": log["total"]}
    dp.close()
    return out



class ClockSampler:
    """nvidia-smi samples of this GPU's SM clock and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.05)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[3:7]) if "Active" in v and "Not" not in v})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def reference_arm(args):
    """Run the unmodified reference through its own API, or say why it cannot run."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    reason = None
    if not os.path.isdir(os.path.join(ref, "xnn")):
        reason = "reference not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref)
        try:
            import xnn.gnn.models.mace  # noqa: F401
        except ModuleNotFoundError as exc:
            reason = (f"the reference MACE imports {exc.name!r}, which is not installed and not in the "
                      "offline wheelhouse (no network); the reference cannot build the benchmarked model")
        except Exception as exc:  # pragma: no cover
            reason = f"reference import failed: {exc!r}"
    if reason is None:
        reason = "reference MACE importable but its arm is not wired"
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from xnn_b200.config import from_dict
    from xnn_b200.data import AtomicDataset, synthetic
    from xnn_b200.parallel import distributed as D
    from xnn_b200.train import Trainer

    world = D.env_world()
    rank = D.env_rank()
    dtype = getattr(torch, args.dtype)
    torch.set_default_dtype(dtype)
    B = args.batch
    # synthetic data: a pool of distinct batches per rank, cycled through the steps
    mols = synthetic.organic_molecules(B * args.pool, seed=1000 + rank)
    ds = AtomicDataset(mols, 4.5, precompute=True)
    graphs = [ds[i] for i in range(len(ds))]
    n_edges = sum(g.num_edges for g in graphs)
    n_atoms = sum(g.num_nodes for g in graphs)
    avg_nb = n_edges / n_atoms
    cfg = from_dict({
        "model": {"name": "mace", "cutoff": 4.5, "n_features": 96, "n_interactions": 2, "n_rbf": 8,
                  "extra": {"species": [1, 6, 7, 8, 9, 16, 17], "max_ell": 3, "max_L": 0,
                            "correlation": 3, "avg_num_neighbors": avg_nb}},
        "optim": {"lr": 1e-3, "energy_weight": 1.0, "force_weight": 10.0, "epochs": 1,
                  "scheduler": "none"},
        "data": {"batch_size": B, "val_fraction": 0.0},
        "trainer": {"cuda_graph": not args.no_graph, "grad_sync": args.grad_sync, "loggers": []},
        "device": "cuda", "seed": 1234, "output_dir": tempfile.mkdtemp(prefix="xnn_b200_bench_"),
    })
    trainer = Trainer(cfg, ds, val=[], test=[])
    dev = trainer.device
    # fixed-capacity padded batches in pinned host memory
    cap = trainer.capacity_for_batches([graphs[k * B:(k + 1) * B] for k in range(args.pool)])
    if world > 1:
        t = torch.tensor(cap, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        cap = tuple(int(x) for x in t.tolist())
    padder = trainer.make_padder(*cap)
    from xnn_b200.data import collate
    host_batches = []
    for k in range(args.pool):
        gs = graphs[k * B:(k + 1) * B]
        host_batches.append(padder(gs) if not args.no_graph else collate(gs).pin_memory())
    in_bytes = [sum(v.numel() * v.element_size() for v in vars(b).values() if isinstance(v, torch.Tensor))
                for b in host_batches]
    dev_batches = [b.to(dev) for b in host_batches]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def step(i, batch):
        return trainer.train_step(batch)

    # warm-up (the first step captures the graph)
    for i in range(max(3, args.warmup)):
        loss, _ = step(i, dev_batches[i % args.pool])
    torch.cuda.synchronize(dev)
    finite = bool(torch.isfinite(loss).item())

    # launch count of this repository's kernels in one step (eager step under the profiler, untimed)
    launches = None
    try:
        from torch.profiler import ProfilerActivity, profile
        trainer.use_graphs, saved = False, trainer.use_graphs
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            trainer._train_step_impl(dev_batches[0])
            torch.cuda.synchronize(dev)
        trainer.use_graphs = saved
        names = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
        ours = [n for n in names if any(k in n for k in OUR_KERNELS)]
        launches = len(ours)
        all_kernels = len(names)
    except Exception as exc:  # pragma: no cover
        all_kernels = None
        print(f"launch count unavailable: {exc}", file=sys.stderr)

    # device-timed region
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record()
            step(i, dev_batches[i % args.pool])
            stops[i].record()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, stops)) / args.steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * B / (ms_max / 1e3)

    # end to end through the public step: pinned host batch in, loss out, every step
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(args.steps):
        loss, _ = trainer.train_step(host_batches[i % args.pool])
        _ = float(loss.item())
    torch.cuda.synchronize(dev)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = world * B * args.steps / float(te.item())

    trainer.close()
    md = None
    if args.md_atoms > 0:
        del dev_batches, flush
        torch.cuda.empty_cache()
        with ClockSampler(torch.cuda.current_device()) as md_clocks:
            md = md_measure(args, dev, world, rank)
        md["clocks"] = md_clocks.summary()
    pme = None
    if args.pme_atoms > 0:
        torch.cuda.empty_cache()
        with ClockSampler(torch.cuda.current_device()) as pme_clocks:
            pme = pme_measure(args, dev, world, rank)
        pme["clocks"] = pme_clocks.summary()
    if rank == 0:
        line = {
            "metric": "MACE train structures/s", "value": round(value, 2), "unit": "structures/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32" if dtype == torch.float32 else str(dtype),
            "data": "synthetic (seeded organic molecules, 10-60 atoms, float64 Morse labels); random-init weights",
            "config": {"model": "MACE OFF23-small-shaped: 2 interactions, 96x0e, max_ell 3, max_L 0, "
                                "correlation 3, 8 Bessel, r_max 4.5 A",
                       "global_batch": world * B, "seq_len": None, "atoms_per_structure": "10-60",
                       "parallelism": f"dp{world}", "grad_sync": args.grad_sync,
                       "cuda_graph": not args.no_graph,
                       "l2": "flushed between timed steps (256 MB write)",
                       "avg_atoms_per_batch": round(n_atoms / args.pool, 1),
                       "avg_edges_per_batch": round(n_edges / args.pool, 1)},
            "clocks": clocks.summary(),
            "e2e": {"value": round(e2e, 2), "unit": "structures/s",
                    "h2d_bytes_per_step": int(sum(in_bytes) / len(in_bytes)), "d2h_bytes_per_step": 8},
            "gpu_launches": None if launches is None else launches * args.steps,
            "gpu_launches_per_step": {"xnn_b200_kernels": launches, "all_kernels": all_kernels},
            "loss_finite": finite,
            "md": md,
            "pme": pme,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
