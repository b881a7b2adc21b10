"""Second-moment-normalised scalar MLPs (e3nn's ``FullyConnectedNet`` layout).

A layer ``h_in -> h_out`` holds ``weight`` of shape ``(h_in, h_out)`` drawn from a unit
normal and computes ``act(x @ W / sqrt(h_in var_in)) * sqrt(var_out)``; the activation
is rescaled so that its second moment under a unit normal input is one. The output
layer has no activation and computes ``x @ W / sqrt(h_in var_in / var_out)``. The
reference's radial networks (``src/xnn/gnn/models/blocks.py:234-290``) fold exactly
these factors, and checkpoints store ``layer{i}.weight``.

The normalising constant is the Monte-Carlo second moment over one million float64
unit normals drawn from a CPU generator seeded with 0, the estimate e3nn uses; an
exact integral would differ from it in the fourth digit, enough to change the
outputs of transplanted weights.
"""
from __future__ import annotations

import functools
from typing import Callable, Optional, Sequence

import torch
from torch import Tensor, nn


@functools.lru_cache(maxsize=None)
def _second_moment_constant(name: str) -> float:
    fn = _NAMED[name]
    gen = torch.Generator(device="cpu").manual_seed(0)
    z = torch.randn(1_000_000, generator=gen, dtype=torch.float64)
    return float(fn(z).pow(2).mean().pow(-0.5))


def _ssp(x: Tensor) -> Tensor:
    import math
    return torch.nn.functional.softplus(x) - math.log(2.0)


_NAMED = {
    "silu": torch.nn.functional.silu,
    "tanh": torch.tanh,
    "abs": torch.abs,
    "ssp": _ssp,
    "sigmoid": torch.sigmoid,
    "gelu": torch.nn.functional.gelu,
    "relu": torch.relu,
    "softplus": torch.nn.functional.softplus,
}


def activation_name(f: Callable) -> Optional[str]:
    for k, v in _NAMED.items():
        if v is f:
            return k
    return None


class normalize2mom(nn.Module):  # noqa: N801 (e3nn's spelling, kept for familiarity)
    """``f`` rescaled to unit second moment under a unit normal input."""

    def __init__(self, f: Callable):
        super().__init__()
        name = activation_name(f)
        if name is not None:
            cst = _second_moment_constant(name)
        else:
            gen = torch.Generator(device="cpu").manual_seed(0)
            z = torch.randn(1_000_000, generator=gen, dtype=torch.float64)
            with torch.no_grad():
                cst = float(f(z).pow(2).mean().pow(-0.5))
        self.f = f
        self.cst = cst
        self._is_id = abs(cst - 1.0) < 1e-4

    def forward(self, x: Tensor) -> Tensor:
        if self._is_id:
            return self.f(x)
        return self.f(x) * self.cst


class _Layer(nn.Module):
    def __init__(self, h_in: int, h_out: int, act, var_in: float, var_out: float):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(h_in, h_out))
        self.act = act
        self.h_in, self.h_out = h_in, h_out
        self.var_in, self.var_out = var_in, var_out

    def scale(self) -> float:
        """Factor on ``x @ W`` before the activation (or the output, without one)."""
        if self.act is not None:
            return (self.h_in * self.var_in) ** -0.5
        return (self.h_in * self.var_in / self.var_out) ** -0.5

    def forward(self, x: Tensor) -> Tensor:
        if self.act is not None:
            x = x @ (self.weight * self.scale())
            x = self.act(x)
            return x * self.var_out ** 0.5
        return x @ (self.weight * self.scale())


class FullyConnectedNet(nn.Sequential):
    """``hs[0] -> hs[1] -> ... -> hs[-1]`` with ``act`` after every hidden layer."""

    def __init__(self, hs: Sequence[int], act: Optional[Callable] = None, variance_in: float = 1.0,
                 variance_out: float = 1.0, out_act: bool = False):
        super().__init__()
        self.hs = tuple(hs)
        if act is not None and not isinstance(act, normalize2mom):
            act = normalize2mom(act)
        var_in = variance_in
        for i, (h1, h2) in enumerate(zip(self.hs, self.hs[1:])):
            last = i == len(self.hs) - 2
            var_out = variance_out if last else 1.0
            a = (act if out_act else None) if last else act
            self.add_module(f"layer{i}", _Layer(h1, h2, a, var_in, var_out))
            var_in = var_out

    def folded(self):
        """Per layer ``(weight, factor, raw activation or None, constant after it)`` such that
        the net equals ``x -> const * f(factor * x @ W)`` applied layer after layer."""
        out = []
        for layer in self:
            act = layer.act
            if act is None:
                out.append((layer.weight, layer.scale(), None, 1.0))
            else:
                f = act.f if isinstance(act, normalize2mom) else act
                cst = 1.0 if (isinstance(act, normalize2mom) and act._is_id) else getattr(act, "cst", 1.0)
                out.append((layer.weight, layer.scale(), f, cst * layer.var_out ** 0.5))
        return out
