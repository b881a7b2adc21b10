"""The Matern kernel of half-integer order ``n + 1/2`` (``n >= 2``) in the form the
gradient-domain fit needs: ``k(r) = exp(-a r) P(r)`` with ``a = sqrt(2n + 1) / sigma`` and
``P(r) = sum_k (n + k)! / (2n)! C(n, k) (2 a r)^(n - k)``, ``g = -k'(r) / r`` and ``t = g'(r) / r``,
each ``exp(-a r)`` times a polynomial (reference ``src/xnn/krnn/kernels.py``). The gradient of
``k(|x - y|)`` with respect to ``x`` is ``-g (x - y)``; the mixed second derivative is
``g I + t d d^T``."""
from __future__ import annotations

import math
from typing import List

import torch
from torch import Tensor


def _polyval(coef: List[float], r: Tensor) -> Tensor:
    out = torch.full_like(r, coef[-1])
    for c in reversed(coef[:-1]):
        out = out * r + c
    return out


def _derivative(coef: List[float]) -> List[float]:
    return [k * c for k, c in enumerate(coef)][1:] or [0.0]


class Matern:
    def __init__(self, sigma: float, n: int = 2):
        self.sigma, self.n = float(sigma), int(n)
        if self.n < 2:
            raise ValueError("the gradient-domain kernel needs a Matern order of at least 5/2 (n >= 2)")
        a = math.sqrt(2 * self.n + 1) / self.sigma
        self.a = a
        f = math.factorial
        p = [0.0] * (self.n + 1)
        for k in range(self.n + 1):
            p[self.n - k] = f(self.n + k) / f(2 * self.n) * math.comb(self.n, k) * (2 * a) ** (self.n - k)
        self.p = p
        q = [a * c for c in p]                      # -k' = exp(-ar) (a P - P')
        for k, c in enumerate(_derivative(p)):
            q[k] -= c
        self.q = q[1:] or [0.0]                     # divided by r (the constant term vanishes)
        t = [-a * c for c in self.q] + [0.0]        # g' = exp(-ar) (Q' - a Q)
        for k, c in enumerate(_derivative(self.q)):
            t[k] += c
        self.t = t[1:] or [0.0]

    def k(self, r: Tensor) -> Tensor:
        return torch.exp(-self.a * r) * _polyval(self.p, r)

    def g(self, r: Tensor) -> Tensor:
        return torch.exp(-self.a * r) * _polyval(self.q, r)

    def t_of(self, r: Tensor) -> Tensor:
        return torch.exp(-self.a * r) * _polyval(self.t, r)

    def g_and_t(self, r: Tensor):
        e = torch.exp(-self.a * r)
        return e * _polyval(self.q, r), e * _polyval(self.t, r)


def safe_norm(x: Tensor) -> Tensor:
    s = (x * x).sum(-1)
    pos = s > 0
    return torch.where(pos, torch.sqrt(torch.where(pos, s, torch.ones_like(s))), torch.zeros_like(s))
