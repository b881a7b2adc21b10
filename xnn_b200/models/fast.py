"""Fast-path selection: one switch per model between the reference formulas and the kernels.

A model with a fast path keeps the reference's parameters and evaluates them either with the
PyTorch formulas (the canonical form, used for export, the CPU and anything the kernels do not
cover) or with this package's kernels. ``use_fast`` chooses, per evaluation:

* ``False``: always the formulas;
* ``True``: the kernels wherever the model and the input are covered;
* ``"auto"`` (default): the kernels when covered *and* the :class:`AutoPolicy` of the model says
  they pay for this input: a minimum edge count per GPU name and precision (the kernels have a
  fixed cost per call), optionally an upper bound, and CPU thresholds for fast paths with a CPU
  implementation.

:func:`set_use_fast` reaches every model inside a wrapper (forces, dispersion, long range). The
kernels sum in a different order, so results agree with the formulas to rounding (about 1e-6
relative in float32, 1e-14 in float64); :class:`FastPathPrecisionWarning` says so once when a fast
path first runs in float32. Parity: ``src/xnn/common/models/fast.py:41-238`` of the reference.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass, field
from typing import Dict, Optional, Union

import torch
from torch import nn

UseFast = Union[bool, str]


class FastPathPrecisionWarning(UserWarning):
    """A fast path ran in float32: results differ from the formulas at rounding level (~1e-6)."""


_WARNED = {"float32": False}


def warn_float32_once() -> None:
    if not _WARNED["float32"]:
        _WARNED["float32"] = True
        warnings.warn("a fast path (this package's kernels) runs in float32: energies and forces agree with the "
                      "reference formulas to about 1e-6 relative (float64: about 1e-14); use_fast=False gives the "
                      "formulas", FastPathPrecisionWarning, stacklevel=3)


def resolve_use_fast(use_fast: UseFast) -> UseFast:
    if isinstance(use_fast, str):
        if use_fast.lower() != "auto":
            raise ValueError(f"use_fast must be True, False or 'auto', got {use_fast!r}")
        return "auto"
    if isinstance(use_fast, bool):
        return use_fast
    raise TypeError(f"use_fast must be True, False or 'auto', got {type(use_fast).__name__}")


def _lookup(table: Dict[str, int], device: torch.device) -> Optional[int]:
    if not table or device.type != "cuda":
        return None
    name = torch.cuda.get_device_name(device).lower()
    for key, value in table.items():
        if key.lower() in name:
            return int(value)
    return None


@dataclass
class AutoPolicy:
    """When ``"auto"`` takes the kernels: edge-count thresholds per GPU name (substring, first
    match) and precision, with defaults for unlisted GPUs, optional upper bounds, CPU thresholds."""
    min_edges: Dict[str, int] = field(default_factory=dict)
    min_edges_float64: Dict[str, int] = field(default_factory=dict)
    default_min_edges: int = 0
    default_min_edges_float64: int = 0
    max_edges: Dict[str, int] = field(default_factory=dict)
    default_max_edges: Optional[int] = None
    cpu_min_edges: Optional[int] = None

    def threshold(self, device: torch.device, dtype: torch.dtype = torch.float32) -> int:
        f64 = dtype == torch.float64
        hit = _lookup(self.min_edges_float64 if f64 else self.min_edges, device)
        if hit is not None:
            return hit
        return int(self.default_min_edges_float64 if f64 else self.default_min_edges)

    def decide(self, device: torch.device, dtype: torch.dtype, num_edges: int) -> bool:
        if device.type == "cpu":
            return self.cpu_min_edges is not None and num_edges >= self.cpu_min_edges
        if device.type != "cuda" or num_edges < self.threshold(device, dtype):
            return False
        bound = _lookup(self.max_edges, device)
        bound = self.default_max_edges if bound is None else bound
        return bound is None or num_edges < bound


def choose(use_fast: UseFast, covered: bool, policy: Optional[AutoPolicy], device: torch.device,
           dtype: torch.dtype, num_edges: int) -> bool:
    """Whether one evaluation takes the kernels (``covered``: the model and input are supported)."""
    if not covered or use_fast is False:
        return False
    fast = True if use_fast is True else (policy is None or policy.decide(device, dtype, num_edges))
    if fast and dtype == torch.float32:
        warn_float32_once()
    return fast


def set_use_fast(model: nn.Module, use_fast: UseFast) -> nn.Module:
    """Set ``use_fast`` on every model inside ``model`` that has a ``set_use_fast`` method."""
    mode = resolve_use_fast(use_fast)
    for m in model.modules():
        if callable(getattr(m, "set_use_fast", None)):
            m.set_use_fast(mode)
    return model
