"""Throughput of batched NDDO evaluations (energy and forces) on one device.

``python -m xnn_b200.sqm.benchmark --params FILE --molecules 1024 --device cuda`` builds a batch of
perturbed copies of small organic molecules (water, methanol, formaldehyde, methylamine,
N-methylformamide), runs ``--warmup`` untimed evaluations and times ``--repeats`` evaluations with
forces, and prints one JSON line (molecules per second, milliseconds per batch, SCF size).
"""
from __future__ import annotations

import argparse
import json
import time

import torch

from ..data import collate
from ..data.dataset import structure_to_graph
from .nddo import PM3

MOLECULES = {
    "water": ([8, 1, 1], [[0, 0, 0.1173], [0, 0.7572, -0.4692], [0, -0.7572, -0.4692]]),
    "methanol": ([6, 8, 1, 1, 1, 1], [[0, 0, 0], [1.42, 0, 0], [1.75, 0.9, 0], [-0.37, 1.02, 0],
                                      [-0.37, -0.51, 0.89], [-0.37, -0.51, -0.89]]),
    "formaldehyde": ([6, 8, 1, 1], [[0, 0, 0], [0, 0, 1.21], [0, 0.94, -0.58], [0, -0.94, -0.58]]),
    "methylamine": ([6, 7, 1, 1, 1, 1, 1], [[0, 0, 0], [1.47, 0, 0], [-0.36, 1.03, 0], [-0.36, -0.5, 0.89],
                                            [-0.36, -0.5, -0.89], [1.8, 0.5, 0.8], [1.8, 0.5, -0.8]]),
    "nmf": ([6, 8, 7, 1, 6, 1, 1, 1, 1], [[0, 0, 0], [0, 1.22, 0], [1.15, -0.68, 0], [-0.94, -0.56, 0],
                                          [2.45, -0.05, 0], [1.12, -1.69, 0.05], [3.25, -0.8, 0],
                                          [2.55, 0.58, 0.89], [2.55, 0.58, -0.89]]),
}


def make_batch(n: int, seed: int = 0):
    gen = torch.Generator().manual_seed(seed)
    names = sorted(MOLECULES)
    graphs = []
    for i in range(n):
        z, pos = MOLECULES[names[i % len(names)]]
        p = torch.tensor(pos, dtype=torch.float64) + 0.03 * torch.randn(len(z), 3, generator=gen, dtype=torch.float64)
        graphs.append(structure_to_graph({"pos": p, "atomic_numbers": torch.tensor(z)}, cutoff=5.0))
    return collate(graphs)


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--params", required=True)
    ap.add_argument("--molecules", type=int, default=1024)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--repeats", type=int, default=5)
    args = ap.parse_args(argv)
    dev = torch.device(args.device)
    model = PM3(args.params).to(dev)
    data = make_batch(args.molecules).to(dev)

    def run():
        d = data.clone() if hasattr(data, "clone") else data
        d.pos = data.pos.detach().clone().requires_grad_(True)
        out = model(d)
        f = -torch.autograd.grad(out["energy"].sum(), d.pos)[0]
        return out, f

    for _ in range(args.warmup):
        run()
    if dev.type == "cuda":
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.repeats):
            out, f = run()
        stop.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop) / args.repeats
    else:
        t0 = time.perf_counter()
        for _ in range(args.repeats):
            out, f = run()
        ms = (time.perf_counter() - t0) * 1e3 / args.repeats
    res = {"metric": "pm3_molecules_per_s", "value": args.molecules / (ms / 1e3), "ms_per_batch": ms,
           "molecules": args.molecules, "atoms": int(data.pos.shape[0]), "device": str(dev),
           "threads": torch.get_num_threads(), "dtype": "float64"}
    print(json.dumps(res))
    return res


if __name__ == "__main__":
    main()
