"""Training callbacks (``src/xnn/common/train/callbacks.py:51-229``)."""
from __future__ import annotations

import os
from typing import Dict, Optional


class Callback:
    def on_fit_start(self, trainer) -> None: ...
    def on_train_batch_end(self, trainer, loss) -> None: ...
    def on_epoch_end(self, trainer, metrics: Dict[str, float]) -> bool:
        return False
    def on_fit_end(self, trainer) -> None: ...


class ModelCheckpoint(Callback):
    """``best.pt`` when the monitored value improves, ``last.pt`` at the end, ``epoch_N.pt`` every N."""

    def __init__(self, output_dir: str, monitor: str = "val/loss", mode: str = "min", every_n: int = 0):
        self.output_dir, self.monitor, self.mode, self.every_n = output_dir, monitor, mode, every_n
        self.best: Optional[float] = None

    def _better(self, v: float) -> bool:
        if self.best is None:
            return True
        return v < self.best if self.mode == "min" else v > self.best

    def on_epoch_end(self, trainer, metrics) -> bool:
        v = metrics.get(self.monitor, metrics.get("train/loss"))
        if v is not None and self._better(float(v)):
            self.best = float(v)
            trainer.best = self.best
            trainer.save(os.path.join(self.output_dir, "best.pt"))
        if self.every_n and (trainer.epoch + 1) % self.every_n == 0:
            trainer.save(os.path.join(self.output_dir, f"epoch_{trainer.epoch + 1}.pt"))
        return False

    def on_fit_end(self, trainer) -> None:
        trainer.save(os.path.join(self.output_dir, "last.pt"))


class EarlyStopping(Callback):
    def __init__(self, monitor: str = "val/loss", patience: int = 10, min_delta: float = 0.0,
                 mode: str = "min", threshold: Optional[float] = None):
        self.monitor, self.patience, self.min_delta, self.mode = monitor, patience, min_delta, mode
        self.threshold = threshold
        self.best: Optional[float] = None
        self.bad = 0

    def on_epoch_end(self, trainer, metrics) -> bool:
        v = metrics.get(self.monitor)
        if v is None:
            return False
        v = float(v)
        if self.threshold is not None and (v < self.threshold if self.mode == "min" else v > self.threshold):
            return True
        improved = self.best is None or (v < self.best - self.min_delta if self.mode == "min"
                                         else v > self.best + self.min_delta)
        if improved:
            self.best, self.bad = v, 0
        else:
            self.bad += 1
        return self.patience > 0 and self.bad >= self.patience


class ProgressBar(Callback):
    def on_epoch_end(self, trainer, metrics) -> bool:
        from ..parallel import distributed as D
        if D.is_main():
            print(f"epoch {trainer.epoch}: " + " ".join(f"{k}={v:.4g}" for k, v in metrics.items()
                                                       if isinstance(v, float)), flush=True)
        return False
