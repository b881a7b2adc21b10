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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="xnn_b200", choices=["xnn_b200", "reference"])
    ap.add_argument("--batch", type=int, default=64, help="structures per GPU per step")
    ap.add_argument("--pool", type=int, default=8, help="distinct batches per rank, cycled")
    ap.add_argument("--no-graph", action="store_true", help="eager steps instead of one CUDA graph")
    ap.add_argument("--grad-sync", default="p2p", choices=["nccl", "p2p"])
    ap.add_argument("--dtype", default="float32")
    ap.add_argument("--md-atoms", type=int, default=1_000_000, help="atoms of the MD water box (0: skip MD)")
    ap.add_argument("--md-steps", type=int, default=10)
    ap.add_argument("--md-warmup", type=int, default=3)
    ap.add_argument("--md-exchange", default="p2p", choices=["collective", "p2p"])
    ap.add_argument("--md-chunk", type=int, default=4_000_000, help="edges per chunk of the lean force pass")
    ap.add_argument("--pme-atoms", type=int, default=100_000, help="atoms of the config-5 water box (0: skip)")
    ap.add_argument("--pme-steps", type=int, default=3)
    ap.add_argument("--pme-exchange", default="collective", choices=["collective", "p2p"])
    ap.add_argument("--tn-batch", type=int, default=32, help="config-3 crystals per GPU per step (0: skip)")
    ap.add_argument("--tn-steps", type=int, default=10)
    ap.add_argument("--tn-pool", type=int, default=4)
    ap.add_argument("--nq-steps", type=int, default=20, help="config-1 NequIP CPU training steps (0: skip)")
    ap.add_argument("--solve-atoms", type=int, default=100_000,
                    help="atoms of the config-5 induction-solve comparison on one GPU (0: skip)")
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


def _device_time(step, batches, warmup, steps, world):
    """Mean device time of ``steps`` calls of ``step`` (CUDA events on the launching stream, after
    ``warmup`` untimed calls, barrier + synchronize on both sides, max over ranks), in ms."""
    import torch
    import torch.distributed as dist
    for i in range(max(3, warmup)):
        step(batches[i % len(batches)])
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        step(batches[i % len(batches)])
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / steps], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


TN_CONFIG = {"model": {"name": "tensornet", "cutoff": 5.0, "n_features": 64, "n_interactions": 2, "n_rbf": 32,
                       "extra": {"n_elements": 90}},
             "optim": {"lr": 1e-3, "energy_weight": 1.0, "force_weight": 10.0, "stress_weight": 1.0, "epochs": 1,
                       "scheduler": "none"},
             "data": {"val_fraction": 0.0, "test_fraction": 0.0},
             "device": "cuda", "seed": 1234}


def tensornet_measure(args, impl, world, rank):
    """Config 3: TensorNet (MatPES-shaped: 2 layers, 64 channels, 32 RBF, 5 A, 89 elements) training on
    32 periodic triclinic crystals of 8-200 atoms per GPU, energy + force + stress loss, through the
    trainer of the package named by ``impl`` (each arm its own stock training step)."""
    import copy

    import torch

    from xnn_b200.data import synthetic          # structure generator only (plain numpy / torch)
    B = args.tn_batch
    structs = synthetic.triclinic_crystals(B * args.tn_pool, seed=3000 + rank)
    cfgd = copy.deepcopy(TN_CONFIG)
    cfgd["data"]["batch_size"] = B
    cfgd["output_dir"] = tempfile.mkdtemp(prefix="xnn_b200_bench_tn_")
    if impl == "reference":
        from xnn.common.config.loaders import from_dict as ref_from_dict
        from xnn.common.data.dataset import AtomicDataset as RefDataset
        from xnn.common.data.dataset import collate as ref_collate
        from xnn.common.train.trainer import Trainer as RefTrainer
        ds = RefDataset(structs, 5.0)
        trainer = RefTrainer(ref_from_dict(cfgd), ds)
        batches = [ref_collate([ds[k] for k in range(j * B, (j + 1) * B)]).to(trainer.device)
                   for j in range(args.tn_pool)]

        def step(b):
            trainer._step(b, True)            # the reference's training step (fit() runs it per batch)
    else:
        from xnn_b200.config import from_dict
        from xnn_b200.data import AtomicDataset, collate
        from xnn_b200.train import Trainer
        cfgd["trainer"] = {"loggers": [], "grad_sync": args.grad_sync, "cuda_graph": False}
        ds = AtomicDataset(structs, 5.0, precompute=True)
        trainer = Trainer(from_dict(cfgd), ds, val=[], test=[])
        batches = [collate([ds[k] for k in range(j * B, (j + 1) * B)]).to(trainer.device)
                   for j in range(args.tn_pool)]

        def step(b):
            trainer.train_step(b)
    ms = _device_time(step, batches, args.warmup, args.tn_steps, world)
    n_atoms = sum(int(b.num_nodes) for b in batches) / len(batches)
    out = {"metric": "TensorNet train structures/s", "value": round(world * B / (ms / 1e3), 2),
           "unit": "structures/s", "ms_per_step": round(ms, 3), "steps": args.tn_steps, "warmup": max(3, args.warmup),
           "config": {"model": "TensorNet MatPES-shaped: 2 layers, 64 ch, 32 RBF, 5.0 A, 89 elements",
                      "global_batch": world * B, "avg_atoms_per_batch": round(n_atoms, 1),
                      "loss": "energy 1 + forces 10 + stress 1", "dtype": "fp32",
                      "data": "synthetic triclinic crystals 8-200 atoms, Morse labels with virial stress"}}
    if hasattr(trainer, "close"):
        trainer.close()
    return out


NQ_CONFIG = {"model": {"name": "nequip", "cutoff": 5.0, "n_features": 32, "n_interactions": 3, "n_rbf": 8,
                       "extra": {"species": [1, 6, 8], "lmax": 2}},
             "optim": {"lr": 1e-2, "energy_weight": 1.0, "force_weight": 100.0, "epochs": 1, "scheduler": "none"},
             "data": {"val_fraction": 0.0, "test_fraction": 0.0, "batch_size": 5},
             "device": "cpu", "seed": 1234}


def nequip_cpu_measure(args):
    """Config 1 on the CPU: NequIP (species H, C, O; l_max 2; 3 layers; 32 channels; 8 Bessel; 5 A)
    trained on the 250 seeded 21-atom molecules in batches of 5, energy + force MSE (force weight 100),
    one process (wall clock: no device). Timed: ``--nq-steps`` training steps after warm-up."""
    import torch

    from xnn_b200.config import from_dict
    from xnn_b200.data import AtomicDataset, collate, synthetic
    from xnn_b200.train import Trainer
    structs = synthetic.small_organic(250, seed=0)
    cfgd = {k: (dict(v) if isinstance(v, dict) else v) for k, v in NQ_CONFIG.items()}
    cfgd["output_dir"] = tempfile.mkdtemp(prefix="xnn_b200_bench_nq_")
    cfgd["trainer"] = {"loggers": [], "cuda_graph": False}
    ds = AtomicDataset(structs, 5.0, precompute=True)
    trainer = Trainer(from_dict(cfgd), ds, val=[], test=[])
    B = 5
    batches = [collate([ds[k] for k in range(j * B, (j + 1) * B)]) for j in range(len(structs) // B)]
    for j in range(max(3, args.warmup)):
        trainer.train_step(batches[j % len(batches)])
    t0 = time.perf_counter()
    for j in range(args.nq_steps):
        trainer.train_step(batches[j % len(batches)])
    dt = time.perf_counter() - t0
    if hasattr(trainer, "close"):
        trainer.close()
    return {"metric": "NequIP train structures/s (CPU)", "value": round(args.nq_steps * B / dt, 2),
            "unit": "structures/s", "ms_per_step": round(1e3 * dt / args.nq_steps, 3), "steps": args.nq_steps,
            "device": "cpu", "threads": torch.get_num_threads(),
            "config": {"model": "NequIP small: species [1, 6, 8], l_max 2, 3 layers, 32 channels, 8 Bessel, 5.0 A",
                       "global_batch": B, "data": "synthetic 21-atom molecules (8 H, 9 C, 4 O), Morse labels",
                       "loss": "energy 1 + forces 100", "dtype": "fp32", "timing": "wall clock"}}


def solve_measure(args, impl):
    """Config 5's hot loop on one GPU: the induced dipoles of the 100,000-atom water box,
    ``(1/alpha - T) mu = F`` solved by preconditioned CG to 1e-5 D, ``T`` the Ewald dipole field
    (real space within 7 A, Thole-damped, a = 0.39, pairs of one molecule excluded; PME 128^3,
    order 5, alpha 0.4; self term). The right-hand side ``F`` is a seeded random field, identical
    for both arms. Timed: pair search, operator setup and the whole solve, each arm on its own
    code (the reference: ``unique_pairs``, the Ewald and Thole ladders, ``MeshPlan`` and ``_pcg``)."""
    import torch

    from xnn_b200.ffnn.water import multipole_water    # the box: positions, molecules, polarizabilities
    dev = torch.device("cuda", torch.cuda.current_device())
    w = multipole_water(args.solve_atoms, seed=0, device=dev)
    pos, cell, pol, mol = w["pos"], w["cell"], w["pol"], w["molecule"]
    n = pos.shape[0]
    g = torch.Generator(device="cpu").manual_seed(5)
    F = (0.05 * torch.randn(n, 3, generator=g, dtype=torch.float64)).to(dev)
    alpha, thole, cutoff, tol = 0.4, 0.39, 7.0, 1e-5
    if impl == "reference":
        from xnn.common.data.neighborlist import unique_pairs
        from xnn.ffnn.models.amoeba import _pcg, coulomb_ladder, mutual_field_real, thole_ladder
        from xnn.ffnn.models.amoeba_ewald import MeshPlan, ewald_ladder, self_field_coefficient
        pbc = torch.ones(3, dtype=torch.bool, device=dev)

        def run():
            i, k, sh = unique_pairs(pos, cutoff, cell, pbc)
            r = pos[k] - pos[i] + sh.to(pos.dtype) @ cell
            R = r.norm(dim=-1)
            De = ewald_ladder(R, torch.full_like(R, alpha), 2)
            th = torch.full_like(R, thole)
            Dt = thole_ladder(R, pol[i], pol[k], th, th, 2)
            Dc = coulomb_ladder(R, 2)
            same = mol[i] == mol[k]
            D1 = De[1] + torch.where(same, -Dc[1], Dt[1] - Dc[1])
            D2 = De[2] + torch.where(same, -Dc[2], Dt[2] - Dc[2])
            ik, ki = torch.cat([i, k]), torch.cat([k, i])
            plan = MeshPlan(pos, cell[None], torch.zeros(n, dtype=torch.long, device=dev), [128] * 3, 5)
            coef = float(self_field_coefficient(alpha))

            def field_of(v, guard=None):
                _, dphi, _ = plan.potential(None, v, None, alpha, hessian=False)
                return mutual_field_real(v, r, D1, D2, ik, ki, n) - dphi + coef * v

            mu, iters = _pcg(F, pol, field_of, torch.ones(n, dtype=torch.bool, device=dev), tol, 100)[:2]
            return mu, iters
    else:
        from xnn_b200.ffnn import multipoles as MP
        setup = MP.EwaldSetup(alpha=alpha, cutoff=cutoff, mesh=(128, 128, 128), order=5, fft_dtype=torch.float32)
        mod = MP.PolarizableMultipoles(setup, tol_debye=tol, max_iter=100, thole=thole)

        def run():
            pairs = mod.pairs(pos, cell, mol)
            mu, iters, _ = mod.solve(pos, cell, pairs, F, pol)
            return mu, iters
    with torch.no_grad():
        mu, iters = run()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        steps = 3
        for _ in range(steps):
            mu, iters = run()
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    return {"metric": "induced-dipole solves/s (100k-atom water box, PME 128^3)", "value": round(1e3 / ms, 3),
            "unit": "solves/s", "ms_per_solve": round(ms, 2), "iterations": int(iters), "steps": steps, "warmup": 1,
            "mu_rms_debye": float((mu * mu).sum(-1).mean().sqrt()) * 4.80320427,
            "config": {"atoms": n, "mesh": [128, 128, 128], "order": 5, "alpha": alpha, "cutoff_A": cutoff,
                       "thole": thole, "tol_debye": tol,
                       "precision": "fp64 real space, fp32 FFT" if impl != "reference" else
                       "fp64 throughout (the reference mesh follows the positions' dtype)",
                       "convergence": "rms preconditioned residual" if impl != "reference" else
                       "rms dipole change per iteration"}}


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
    """Run the unmodified reference through its own API, or say why it cannot.

    The headline model (MACE) needs ``e3nn``, which is absent offline, so the headline arm prints
    ``unavailable``; the same line carries the configs the reference can run on this box: TensorNet
    training (config 3) and the induced-dipole solve of config 5 (one GPU: the reference PME has no
    multi-GPU path)."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    reason = None
    extra = {}
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if not os.path.isdir(os.path.join(ref, "xnn")):
        reason = "reference not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref)
        sys.path.insert(1, ROOT)
        try:
            import xnn.gnn.models.mace  # noqa: F401
        except ModuleNotFoundError as exc:
            reason = (f"the reference MACE imports {exc.name!r}, which is not installed and not in the "
                      "offline wheelhouse (no network); the reference cannot build the benchmarked model")
        except Exception as exc:  # pragma: no cover
            reason = f"reference import failed: {exc!r}"
        import torch
        if torch.cuda.is_available():
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
            if args.tn_batch > 0:
                try:
                    extra["tensornet"] = tensornet_measure(args, "reference", world, rank)
                except Exception as exc:  # pragma: no cover
                    extra["tensornet"] = {"unavailable": f"reference TensorNet run failed: {exc!r}"[:300]}
            if args.nq_steps > 0 and world == 1:
                extra["nequip_cpu"] = {"unavailable": "the reference NequIP imports e3nn, which is not installed and "
                                                      "not in the offline wheelhouse"}
            if args.solve_atoms > 0:
                if world == 1:
                    try:
                        extra["solve"] = solve_measure(args, "reference")
                    except Exception as exc:  # pragma: no cover
                        extra["solve"] = {"unavailable": f"reference solve failed: {exc!r}"[:300]}
                else:
                    extra["solve"] = {"unavailable": "the reference PME runs on one GPU only"}
    if reason is None:
        reason = "reference MACE importable but its arm is not wired"
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason, **extra}), flush=True)
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


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
        names = [e.name for e in prof.events()
                 if e.device_type.name == "CUDA" and not getattr(e, "is_user_annotation", False)]
        from xnn_b200.utils.profiling import is_own_kernel
        ours = [n for n in names if is_own_kernel(n)]
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
    tn = None
    if args.tn_batch > 0:
        torch.cuda.empty_cache()
        tn = tensornet_measure(args, "xnn_b200", world, rank)
    solve = None
    if args.solve_atoms > 0 and world == 1:
        torch.cuda.empty_cache()
        solve = solve_measure(args, "xnn_b200")
    nequip = None
    if args.nq_steps > 0 and world == 1:
        nequip = nequip_cpu_measure(args)
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
            "tensornet": tn,
            "solve": solve,
            "nequip_cpu": nequip,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
