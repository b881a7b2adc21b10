"""Console / CSV / TensorBoard loggers, rank 0 only (``src/xnn/common/train/loggers.py``)."""
from __future__ import annotations

import csv
import os
from typing import Dict, List

UNITS = {"energy": "eV/atom", "forces": "eV/A", "stress": "eV/A^3"}


class Logger:
    def log(self, metrics: Dict[str, float], step: int) -> None: ...
    def close(self) -> None: ...


class ConsoleLogger(Logger):
    def log(self, metrics, step):
        parts = []
        for k, v in metrics.items():
            if isinstance(v, float):
                unit = next((u for q, u in UNITS.items() if q in k and ("mae" in k or "rmse" in k)), "")
                parts.append(f"{k}={v:.5g}{(' ' + unit) if unit else ''}")
        print(f"[step {step}] " + " | ".join(parts), flush=True)


class CSVLogger(Logger):
    def __init__(self, output_dir: str):
        os.makedirs(output_dir, exist_ok=True)
        self.path = os.path.join(output_dir, "metrics.csv")
        self.keys: List[str] = []

    def log(self, metrics, step):
        row = {"step": step, **{k: v for k, v in metrics.items() if isinstance(v, (int, float))}}
        new = [k for k in row if k not in self.keys]
        if new:
            self.keys += new
            rows = []
            if os.path.exists(self.path):
                with open(self.path) as f:
                    rows = list(csv.DictReader(f))
            with open(self.path, "w", newline="") as f:
                w = csv.DictWriter(f, fieldnames=self.keys)
                w.writeheader()
                for r in rows:
                    w.writerow(r)
                w.writerow(row)
        else:
            with open(self.path, "a", newline="") as f:
                csv.DictWriter(f, fieldnames=self.keys).writerow(row)


class TensorBoardLogger(Logger):
    def __init__(self, output_dir: str):
        try:
            from torch.utils.tensorboard import SummaryWriter
        except Exception as exc:  # pragma: no cover - optional dependency
            raise ImportError("TensorBoardLogger needs tensorboard") from exc
        self.w = SummaryWriter(output_dir)

    def log(self, metrics, step):
        for k, v in metrics.items():
            if isinstance(v, (int, float)):
                self.w.add_scalar(k, v, step)

    def close(self):
        self.w.close()


def make_loggers(cfg) -> List[Logger]:
    out: List[Logger] = []
    for name in cfg.trainer.loggers:
        if name == "console":
            out.append(ConsoleLogger())
        elif name == "csv":
            out.append(CSVLogger(cfg.output_dir))
        elif name == "tensorboard":
            out.append(TensorBoardLogger(cfg.output_dir))
        else:
            raise ValueError(f"unknown logger {name!r}")
    return out
