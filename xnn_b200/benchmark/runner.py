"""Benchmark runner: predictions of a model on labelled structures and their error metrics.

Capabilities follow the reference's ``src/xnn/common/benchmark`` (``runner.py:57-615``,
``metrics.py:165-331``): MAE / RMSE / max error of energies (total and per atom), forces
(component-wise) and stresses, reported as JSON, CSV or Markdown; under ``torchrun`` the
structures are sharded round-robin over the ranks and the predictions gathered.
"""
from __future__ import annotations

import json
import math
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..data.dataset import collate, structure_to_graph


def evaluate_structures(model, structures: List[dict], cutoff: float, batch_size: int = 16,
                        device: str = "cpu") -> List[Dict[str, torch.Tensor]]:
    """Per-structure predictions (energy, forces, stress when present) in input order."""
    world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
    rank = dist.get_rank() if world > 1 else 0
    mine = list(range(rank, len(structures), world))
    preds: Dict[int, Dict[str, torch.Tensor]] = {}
    model = model.to(device)
    for b0 in range(0, len(mine), batch_size):
        idx = mine[b0:b0 + batch_size]
        graphs = [structure_to_graph(structures[i], cutoff) for i in idx]
        batch = collate(graphs).to(device)
        out = model(batch)
        counts = torch.bincount(batch.batch, minlength=len(idx)).tolist()
        starts = [0]
        for c in counts[:-1]:
            starts.append(starts[-1] + c)
        for j, i in enumerate(idx):
            p = {"energy": out["energy"][j].detach().double().cpu(), "n_atoms": torch.tensor(counts[j])}
            if "forces" in out:
                p["forces"] = out["forces"][starts[j]:starts[j] + counts[j]].detach().double().cpu()
            if "stress" in out and structures[i].get("cell") is not None:
                p["stress"] = out["stress"][j].detach().double().cpu()
            preds[i] = p
    if world > 1:
        parts = [None] * world
        dist.all_gather_object(parts, preds)
        preds = {k: v for part in parts for k, v in part.items()}
    return [preds[i] for i in range(len(structures))]


def _stats(err: torch.Tensor) -> Dict[str, float]:
    if err.numel() == 0:
        return {"mae": math.nan, "rmse": math.nan, "max": math.nan, "n": 0}
    e = err.double().abs()
    return {"mae": float(e.mean()), "rmse": float(e.square().mean().sqrt()), "max": float(e.max()), "n": int(err.numel())}


def error_report(structures: List[dict], preds: List[Dict[str, torch.Tensor]]) -> Dict[str, Dict[str, float]]:
    de, dea, df, ds = [], [], [], []
    for s, p in zip(structures, preds):
        if s.get("energy") is not None:
            d = p["energy"] - float(s["energy"])
            de.append(d.reshape(1))
            dea.append((d / p["n_atoms"]).reshape(1))
        if s.get("forces") is not None and "forces" in p:
            df.append((p["forces"] - torch.as_tensor(s["forces"]).double()).reshape(-1))
        if s.get("stress") is not None and "stress" in p:
            ds.append((p["stress"] - torch.as_tensor(s["stress"]).double().reshape(3, 3)).reshape(-1))
    cat = lambda xs: torch.cat(xs) if xs else torch.zeros(0)  # noqa: E731
    return {"energy": _stats(cat(de)), "energy_per_atom": _stats(cat(dea)), "forces": _stats(cat(df)),
            "stress": _stats(cat(ds))}


def format_report(report: Dict[str, Dict[str, float]], fmt: str = "json") -> str:
    if fmt == "json":
        return json.dumps(report, indent=2)
    rows = [(k, v["mae"], v["rmse"], v["max"], v["n"]) for k, v in report.items()]
    if fmt == "csv":
        return "quantity,mae,rmse,max,n\n" + "\n".join(f"{a},{b:.6g},{c:.6g},{d:.6g},{e}" for a, b, c, d, e in rows)
    if fmt in ("md", "markdown"):
        head = "| quantity | MAE | RMSE | max | n |\n|---|---|---|---|---|\n"
        return head + "\n".join(f"| {a} | {b:.6g} | {c:.6g} | {d:.6g} | {e} |" for a, b, c, d, e in rows)
    raise ValueError(f"unknown report format {fmt!r}")


def run_benchmark(model_source: str, data_path: str, batch_size: int = 16, device: str = "cpu",
                  fmt: str = "json", out: Optional[str] = None) -> Dict[str, Dict[str, float]]:
    from ..data.io import read_structures
    from ..hub import from_pretrained
    model = from_pretrained(model_source)
    structures = read_structures(data_path)
    preds = evaluate_structures(model, structures, float(model.cutoff), batch_size, device)
    report = error_report(structures, preds)
    if out is not None and (not dist.is_initialized() or dist.get_rank() == 0):
        with open(out, "w") as f:
            f.write(format_report(report, fmt) + "\n")
    return report
