"""``xnn_b200`` command line, the verbs of the reference's ``xnn`` CLI (``src/xnn/common/cli/main.py``).

* ``train --config run.yaml [--set key=value ...]``: build the data sets named by
  ``data.train_path`` / ``val_path`` / ``test_path`` (extxyz, RuNNer, ``.pt``; or
  ``synthetic:<organic|crystals|water>:<count>``) and run ``Trainer(cfg, data).fit()``; under
  ``torchrun`` every process joins the data-parallel run;
* ``benchmark --model M --data FILE [--format json|csv|md] [--out FILE]``: error metrics;
  ``benchmark --suite FILE [--models A,B | --shard I/N | --parallel [K] | --merge]``: several models;
* ``export --model M --format lammps|torchscript --out FILE``;
* ``mdi --model M --mdi "<MDI options>"``: serve the model as an MDI engine;
* ``models``: registered architectures and locally registered pretrained models.
"""
from __future__ import annotations

import argparse
import json
import sys
from typing import List, Optional


def _structures(spec: Optional[str], seed: int):
    if not spec:
        return None
    if spec.startswith("synthetic:"):
        from ..data import synthetic
        _, kind, count = spec.split(":")
        n = int(count)
        if kind == "organic":
            return synthetic.organic_molecules(n, seed=seed)
        if kind == "crystals":
            return synthetic.triclinic_crystals(n, seed=seed)
        if kind == "small":
            return synthetic.small_organic(n, seed=seed)
        raise ValueError(f"unknown synthetic data set {kind!r}")
    from ..data.io import read_structures
    return read_structures(spec)


def cmd_train(args) -> int:
    from ..config import from_argparse
    from ..data import AtomicDataset
    from ..train import Trainer
    cfg = from_argparse(args)
    cut = float(cfg.model.cutoff)
    train = AtomicDataset(_structures(cfg.data.train_path, cfg.seed), cut)
    val = _structures(cfg.data.val_path, cfg.seed + 1)
    test = _structures(cfg.data.test_path, cfg.seed + 2)
    trainer = Trainer(cfg, train, val=AtomicDataset(val, cut) if val else None,
                      test=AtomicDataset(test, cut) if test else None)
    try:
        metrics = trainer.fit()
    finally:
        trainer.close()
    print(json.dumps({k: float(v) for k, v in (metrics or {}).items()}))
    return 0


def cmd_benchmark(args) -> int:
    if args.suite:
        from ..benchmark import suite as S
        if args.parallel is not None:
            rows = S.run_parallel(args.suite, args.parallel)
        else:
            cfg = S.load_suite(args.suite)
            if args.device:
                cfg["device"] = args.device
            if args.merge:
                rows = S.merge_parts(cfg)
            else:
                entries = S.select_entries(cfg, args.models, args.shard)
                rows = S.score(cfg, entries)
                S.write_part(cfg, rows, entries)
                if args.models is None and args.shard is None:
                    S.write_table(cfg, rows)
        print(json.dumps(rows, indent=1))
        return 0
    if not args.model or not args.data:
        raise SystemExit("benchmark needs --model and --data, or --suite")
    from ..benchmark import format_report, run_benchmark
    report = run_benchmark(args.model, args.data, args.batch_size, args.device or "cpu", args.format, args.out)
    print(format_report(report, args.format))
    return 0


def cmd_export(args) -> int:
    from ..hub import from_pretrained
    model = from_pretrained(args.model)
    if args.format == "lammps":
        from ..deploy.lammps import export_to_lammps
        export_to_lammps(model, args.cutoff, args.out)
    else:
        from ..deploy.torchscript import export_torchscript
        export_torchscript(model, args.out)
    print(args.out)
    return 0


def cmd_mdi(args) -> int:  # pragma: no cover - needs an MDI driver
    from ..deploy.mdi_engine import MDIEngine, mdi_comm
    from ..hub import from_pretrained
    MDIEngine(from_pretrained(args.model), device=args.device).serve(mdi_comm(args.mdi))
    return 0


def cmd_models(args) -> int:
    from ..hub import list_pretrained
    from ..models import list_models
    print(json.dumps({"architectures": sorted(list_models()),
                      "pretrained": {k: str(v) for k, v in list_pretrained().items()}}, indent=2))
    return 0


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="xnn_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    t = sub.add_parser("train")
    t.add_argument("--config")
    t.add_argument("--set", action="append", default=[])
    t.set_defaults(fn=cmd_train)
    b = sub.add_parser("benchmark")
    b.add_argument("--model")
    b.add_argument("--data")
    b.add_argument("--suite", help="a suite YAML of several models (see xnn_b200.benchmark.suite)")
    b.add_argument("--models", help="suite: labels or positions to score, comma separated")
    b.add_argument("--shard", help="suite: I/N (every N-th model from I) or 'slurm'")
    b.add_argument("--parallel", type=int, nargs="?", const=0, default=None,
                   help="suite: one worker per model, this many at once (default: one per visible GPU)")
    b.add_argument("--merge", action="store_true", help="suite: assemble the part files into the table")
    b.add_argument("--batch-size", type=int, default=16)
    b.add_argument("--device", default=None)
    b.add_argument("--format", default="json", choices=["json", "csv", "md"])
    b.add_argument("--out")
    b.set_defaults(fn=cmd_benchmark)
    e = sub.add_parser("export")
    e.add_argument("--model", required=True)
    e.add_argument("--format", default="lammps", choices=["lammps", "torchscript"])
    e.add_argument("--cutoff", type=float)
    e.add_argument("--out", required=True)
    e.set_defaults(fn=cmd_export)
    m = sub.add_parser("mdi")
    m.add_argument("--model", required=True)
    m.add_argument("--mdi", required=True)
    m.add_argument("--device", default="cpu")
    m.set_defaults(fn=cmd_mdi)
    sub.add_parser("models").set_defaults(fn=cmd_models)
    return ap


def main(argv: Optional[List[str]] = None) -> int:
    args = build_parser().parse_args(argv)
    return args.fn(args)


if __name__ == "__main__":
    sys.exit(main())
