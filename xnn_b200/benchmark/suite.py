"""Benchmark suites: several models scored on one data set, split over runs or worker processes.

A suite file (YAML) names the models and the data::

    models:
      - {label: schnet-small, model: runs/schnet/best}      # any source from_pretrained takes
      - {label: mace-off, model: doi:10.5281/zenodo.123}
    data: data/test.extxyz
    batch_size: 16
    device: cuda
    output: {dir: bench_out, filename: results, formats: [json, md]}

* :func:`select_entries` picks the models one run scores: by label or position (``models``),
  and/or every ``N``-th from ``I`` (``shard="I/N"``; ``"slurm"`` reads ``I`` and ``N`` from the job
  array variables), so a job array covers the suite;
* each run writes its rows to ``<dir>/parts/<filename>.<labels>.json`` and :func:`merge_parts`
  assembles the table in suite order (a model without a part is reported and left out);
* :func:`run_parallel` does the same within one node: one worker process per model, at most
  ``workers`` at a time, each pinned to one GPU through ``CUDA_VISIBLE_DEVICES`` (worker ``k`` on the
  ``k``-th visible GPU, cycling), logs in ``parts/<label>.log``, then the merge.

Parity: ``src/xnn/common/benchmark/runner.py:456-660`` of the reference (``--models``, ``--shard``,
parts and merge, ``--parallel``).
"""
from __future__ import annotations

import json
import os
import re
import subprocess
import sys
import time
from typing import Dict, List, Optional, Sequence, Union

PARTS_DIR = "parts"


def load_suite(path_or_dict: Union[str, dict]) -> dict:
    if isinstance(path_or_dict, dict):
        cfg = dict(path_or_dict)
    else:
        import yaml
        with open(path_or_dict) as f:
            cfg = yaml.safe_load(f) or {}
    models = cfg.get("models") or []
    if not models:
        raise ValueError("a suite needs a non-empty 'models' list")
    entries = []
    for k, m in enumerate(models):
        m = {"model": m} if isinstance(m, str) else dict(m)
        m.setdefault("label", os.path.basename(str(m["model"]).rstrip("/")) or f"model{k}")
        entries.append(m)
    labels = [e["label"] for e in entries]
    if len(set(labels)) != len(labels):
        raise ValueError(f"model labels must be unique: {labels}")
    cfg["models"] = entries
    if "data" not in cfg:
        raise ValueError("a suite needs 'data' (a structure file)")
    out = dict(cfg.get("output") or {})
    out.setdefault("dir", "bench_out")
    out.setdefault("filename", "results")
    out.setdefault("formats", ["json"])
    cfg["output"] = out
    cfg.setdefault("batch_size", 16)
    cfg.setdefault("device", "cpu")
    return cfg


def select_entries(cfg: dict, models: Union[None, str, Sequence[str]] = None, shard: Optional[str] = None) -> List[dict]:
    entries = list(cfg["models"])
    if models is not None:
        wanted = [m.strip() for m in (models.split(",") if isinstance(models, str) else models) if m.strip()]
        by_label = {e["label"]: e for e in entries}
        picked = []
        for m in wanted:
            if m in by_label:
                picked.append(by_label[m])
            elif m.isdigit() and int(m) < len(entries):
                picked.append(entries[int(m)])
            else:
                raise ValueError(f"unknown model {m!r}; the suite has {list(by_label)}")
        entries = picked
    if shard is not None:
        if shard.strip().lower() == "slurm":
            env = os.environ
            if "SLURM_ARRAY_TASK_ID" not in env:
                raise ValueError("shard 'slurm' needs a job array (SLURM_ARRAY_TASK_ID unset)")
            i = int(env["SLURM_ARRAY_TASK_ID"]) - int(env.get("SLURM_ARRAY_TASK_MIN", "0"))
            n = int(env["SLURM_ARRAY_TASK_COUNT"])
        else:
            m = re.fullmatch(r"\s*(\d+)\s*/\s*(\d+)\s*", shard)
            if m is None:
                raise ValueError(f"shard must be I/N or 'slurm', got {shard!r}")
            i, n = int(m.group(1)), int(m.group(2))
        if not 0 <= i < n:
            raise ValueError(f"shard index {i} outside 0..{n - 1}")
        entries = entries[i::n]
    return entries


def _tag(entries: List[dict]) -> str:
    return "+".join(re.sub(r"[^\w.\-#]+", "_", e["label"]) for e in entries)


def _parts(cfg: dict) -> str:
    return os.path.join(cfg["output"]["dir"], PARTS_DIR)


def score(cfg: dict, entries: List[dict]) -> List[dict]:
    """One row per entry: the model's error report on the suite's data."""
    from .runner import run_benchmark
    rows = []
    for e in entries:
        t0 = time.perf_counter()
        rep = run_benchmark(str(e["model"]), str(cfg["data"]), int(cfg["batch_size"]), str(cfg["device"]))
        row = {"model": e["label"], "seconds": round(time.perf_counter() - t0, 3)}
        for q, st in rep.items():
            for k, v in st.items():
                row[f"{q}_{k}"] = v
        rows.append(row)
    return rows


def write_part(cfg: dict, rows: List[dict], entries: List[dict]) -> str:
    os.makedirs(_parts(cfg), exist_ok=True)
    path = os.path.join(_parts(cfg), f"{cfg['output']['filename']}.{_tag(entries)}.json")
    with open(path, "w") as f:
        json.dump(rows, f, indent=1)
    return path


def write_table(cfg: dict, rows: List[dict]) -> List[str]:
    out = cfg["output"]
    os.makedirs(out["dir"], exist_ok=True)
    paths = []
    cols = list(rows[0]) if rows else ["model"]
    for fmt in out["formats"]:
        path = os.path.join(out["dir"], f"{out['filename']}.{fmt}")
        with open(path, "w") as f:
            if fmt == "json":
                json.dump(rows, f, indent=1)
            elif fmt == "csv":
                f.write(",".join(cols) + "\n")
                for r in rows:
                    f.write(",".join(str(r.get(c, "")) for c in cols) + "\n")
            elif fmt in ("md", "markdown"):
                f.write("| " + " | ".join(cols) + " |\n|" + "---|" * len(cols) + "\n")
                for r in rows:
                    f.write("| " + " | ".join(f"{r.get(c, ''):.6g}" if isinstance(r.get(c), float) else str(r.get(c, ""))
                                            for c in cols) + " |\n")
            else:
                raise ValueError(f"unknown output format {fmt!r}")
        paths.append(path)
    return paths


def merge_parts(cfg: dict) -> List[dict]:
    import glob
    files = sorted(glob.glob(os.path.join(_parts(cfg), f"{cfg['output']['filename']}.*.json")))
    if not files:
        raise FileNotFoundError(f"no part files under {_parts(cfg)}")
    found: Dict[str, dict] = {}
    for p in files:
        with open(p) as f:
            for r in json.load(f):
                found[r["model"]] = r
    labels = [e["label"] for e in cfg["models"]]
    missing = [x for x in labels if x not in found]
    if missing:
        print(f"merge: no part for {missing}; left out", file=sys.stderr)
    rows = [found[x] for x in labels if x in found]
    if rows:
        write_table(cfg, rows)
    return rows


def _visible_gpus() -> List[str]:
    env = os.environ.get("CUDA_VISIBLE_DEVICES")
    if env is not None:
        return [d for d in env.split(",") if d.strip()]
    try:
        import torch
        return [str(i) for i in range(torch.cuda.device_count())]
    except Exception:  # pragma: no cover
        return []


def run_parallel(suite_path: str, workers: Optional[int] = None) -> List[dict]:
    """Score every model of the suite in its own worker process (see module notes)."""
    cfg = load_suite(suite_path)
    gpus = _visible_gpus() if str(cfg["device"]).startswith("cuda") else []
    if workers is None or workers <= 0:
        if not gpus:
            raise ValueError("a CPU-only parallel run needs an explicit worker count")
        workers = len(gpus)
    os.makedirs(_parts(cfg), exist_ok=True)
    pending = list(cfg["models"])
    running: List[tuple] = []
    free = list(range(workers))
    failed: List[tuple] = []
    while pending or running:
        while pending and free:
            e = pending.pop(0)
            slot = free.pop(0)
            env = dict(os.environ)
            if gpus:
                env["CUDA_VISIBLE_DEVICES"] = gpus[slot % len(gpus)]
            log = os.path.join(_parts(cfg), re.sub(r"[^\w.\-#]+", "_", e["label"]) + ".log")
            fh = open(log, "w")
            cmd = [sys.executable, "-m", "xnn_b200", "benchmark", "--suite", suite_path, "--models", e["label"]]
            if gpus:
                cmd += ["--device", "cuda"]
            running.append((subprocess.Popen(cmd, stdout=fh, stderr=subprocess.STDOUT, env=env), e, log, fh, slot))
        time.sleep(0.2)
        still = []
        for proc, e, log, fh, slot in running:
            if proc.poll() is None:
                still.append((proc, e, log, fh, slot))
                continue
            fh.close()
            free.append(slot)
            if proc.returncode != 0:
                failed.append((e["label"], log))
        running = still
    if failed:
        raise RuntimeError(f"benchmark workers failed: {failed}")
    return merge_parts(cfg)
