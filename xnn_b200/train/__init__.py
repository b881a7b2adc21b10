"""Training: the Trainer, losses, callbacks, loggers and captured steps."""
from .callbacks import Callback, EarlyStopping, ModelCheckpoint, ProgressBar
from .graphed import GraphedStep, PaddedCollate, pad_graph
from .losses import error_metrics, weighted_loss
from .trainer import EMA, Trainer

__all__ = ["Callback", "EMA", "EarlyStopping", "GraphedStep", "ModelCheckpoint", "PaddedCollate",
           "ProgressBar", "Trainer", "error_metrics", "pad_graph", "weighted_loss"]
