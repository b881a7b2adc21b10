"""Smooth cutoff envelopes (``src/xnn/common/featurizers/cutoff.py:10,44,83``)."""
from __future__ import annotations

import math

import torch
from torch import Tensor, nn


class CosineCutoff(nn.Module):
    """``0.5 (cos(pi r / rc) + 1)`` inside the cutoff, zero outside (Behler / SchNet)."""

    def __init__(self, cutoff: float):
        super().__init__()
        self.cutoff = float(cutoff)

    def forward(self, r: Tensor) -> Tensor:
        return 0.5 * (torch.cos(math.pi * r / self.cutoff) + 1.0) * (r < self.cutoff)


class MollifierCutoff(nn.Module):
    """The C-infinity bump ``exp(1 - 1 / (1 - (r/rc)^2))`` inside the cutoff."""

    def __init__(self, cutoff: float, eps: float = 1e-7):
        super().__init__()
        self.cutoff = float(cutoff)
        self.eps = eps

    def forward(self, r: Tensor) -> Tensor:
        x = (r / self.cutoff).clamp(max=1.0 - self.eps)
        return torch.exp(1.0 - 1.0 / (1.0 - x * x)) * (r < self.cutoff)


class PolynomialCutoff(nn.Module):
    """Degree-``p`` polynomial envelope, 1 at the origin and C^2 to zero at ``rc``:
    ``1 - (p+1)(p+2)/2 x^p + p(p+2) x^(p+1) - p(p+1)/2 x^(p+2)`` with ``x = r / rc``."""

    def __init__(self, cutoff: float, p: int = 6):
        super().__init__()
        self.cutoff = float(cutoff)
        self.p = int(p)

    def forward(self, r: Tensor) -> Tensor:
        x = r / self.cutoff
        p = self.p
        poly = ((-(p * (p + 1) / 2.0)) * x + p * (p + 2.0)) * x - (p + 1) * (p + 2) / 2.0
        return (1.0 + poly * x ** p) * (r < self.cutoff)
