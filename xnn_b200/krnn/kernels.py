"""Half-integer Matern kernels as radial functions, with the derivatives a gradient-domain fit uses.

For order ``nu = n + 1/2`` and length scale ``sigma`` (Rasmussen & Williams, eq. 4.16; Chmiela
et al., Sci. Adv. 3, e1603015, 2017, eq. 3):

    k(r) = exp(-a r) P(r),   a = sqrt(2 nu) / sigma,
    P(r) = sum_{i=0..n} C(n, i) (n + i)! / (2n)! (2 a r)^(n - i).

Force fits differentiate ``k(|x - y|)`` twice in the coordinates, which needs

    g(r) = -k'(r) / r        and        t(r) = g'(r) / r.

Both are ``exp(-a r)`` times a polynomial: with ``k' = exp(-a r) (P' - a P)`` the numerator of
``g`` is ``a P - P'``, whose constant term is zero because ``k`` is flat at the origin; the
numerator of ``t`` is ``Q' - a Q`` for ``Q = (a P - P') / r``, again without a constant term
when ``n >= 2``. The polynomials are built once with :class:`numpy.polynomial.Polynomial`
arithmetic and evaluated by Horner's rule on tensors. Gradient of ``k(|x - y|)`` in ``x``:
``-g(r) (x - y)``; mixed second derivative: ``g I + t d d^T`` with ``d = x - y``.
"""
from __future__ import annotations

import math
from typing import List

import numpy as np
import torch
from numpy.polynomial import Polynomial
from torch import Tensor


def _horner(coef: List[float], r: Tensor) -> Tensor:
    acc = torch.zeros_like(r) + coef[-1]
    for c in coef[-2::-1]:
        acc = torch.addcmul(torch.full_like(r, c), acc, r)
    return acc


def _over_r(poly: Polynomial) -> Polynomial:
    """``poly / r`` for a polynomial whose value at 0 vanishes (its rounding residue is dropped)."""
    c = poly.coef
    return Polynomial(c[1:] if c.size > 1 else np.zeros(1))


class Matern:
    """Matern kernel of order ``n + 1/2`` (``n >= 2``) with length scale ``sigma``."""

    def __init__(self, sigma: float, n: int = 2):
        self.sigma, self.n = float(sigma), int(n)
        if self.n < 2:
            raise ValueError("the gradient-domain kernel needs a Matern order of at least 5/2 (n >= 2)")
        n, a = self.n, math.sqrt(2 * self.n + 1) / self.sigma
        self.a = a
        # P(r): the coefficient of r^(n - i) is C(n, i) (n + i)! / (2n)! (2a)^(n - i)
        coef = np.zeros(n + 1)
        for i in range(n + 1):
            coef[n - i] = math.comb(n, i) * math.factorial(n + i) / math.factorial(2 * n) * (2.0 * a) ** (n - i)
        P = Polynomial(coef)
        Q = _over_r(a * P - P.deriv())
        T = _over_r(Q.deriv() - a * Q)
        self.p, self.q, self.t = (list(map(float, x.coef)) for x in (P, Q, T))

    def _exp(self, r: Tensor) -> Tensor:
        return torch.exp(-self.a * r)

    def k(self, r: Tensor) -> Tensor:
        """``k(r)``."""
        return self._exp(r) * _horner(self.p, r)

    def g(self, r: Tensor) -> Tensor:
        """``-k'(r) / r``."""
        return self._exp(r) * _horner(self.q, r)

    def t_of(self, r: Tensor) -> Tensor:
        """``g'(r) / r``."""
        return self._exp(r) * _horner(self.t, r)

    def g_and_t(self, r: Tensor):
        """``g(r)`` and ``t(r)`` sharing one exponential."""
        e = self._exp(r)
        return e * _horner(self.q, r), e * _horner(self.t, r)


def safe_norm(x: Tensor) -> Tensor:
    """Length over the last axis whose derivative is 0 (not NaN) at the origin; exact for the
    kernels above, whose radial functions are flat at ``r = 0``."""
    sq = x.pow(2).sum(-1)
    nz = sq > 0
    return torch.sqrt(torch.where(nz, sq, torch.ones_like(sq))) * nz.to(sq.dtype)
