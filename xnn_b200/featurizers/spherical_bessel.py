"""Spherical Bessel functions, their zeros, zonal and real spherical harmonics, and the
DimeNet spherical Fourier-Bessel basis.

``j_l(x)``: the power series ``x^l / (2l+1)!! sum_k (-x^2/2)^k / (k! prod_{i=1..k} (2l+2i+1))``
below ``x < l + 2`` (where the upward recurrence loses digits) and the recurrence
``j_{l+1} = (2l+1)/x j_l - j_{l-1}`` from ``sin x / x`` above; both branches are plain tensor
expressions, so autograd differentiates them to any order. Zeros by bisection between the
interlacing zeros of ``j_{l-1}``. The basis ``sqrt(2 / (c^3 j_{l+1}(z_ln)^2)) j_l(z_ln r / c)
Y_l0(alpha)`` follows DimeNet (Gasteiger et al. 2020); buffer names follow the reference
(``src/xnn/gnn/featurizers/spherical_bessel.py``).
"""
from __future__ import annotations

import math
from typing import List

import numpy as np
import torch
from torch import Tensor, nn

_TERMS = 30


def spherical_bessel_jn(l_max: int, x: Tensor, n_terms: int = _TERMS) -> Tensor:
    """``j_0 .. j_{l_max}`` at ``x`` (stacked on a new last axis), computed in float64."""
    x64 = x.to(torch.float64)
    orders = torch.arange(l_max + 1, dtype=torch.float64, device=x.device)
    i = torch.arange(1, n_terms, dtype=torch.float64, device=x.device).unsqueeze(-1)
    coef = torch.cat([torch.ones(1, l_max + 1, dtype=torch.float64, device=x.device),
                      torch.cumprod(1.0 / (i * (2.0 * orders + 2.0 * i + 1.0)), 0)])
    y = (-0.5 * x64 * x64).unsqueeze(-1)
    total = coef[n_terms - 1].expand(list(x64.shape) + [l_max + 1])
    for k in range(n_terms - 2, -1, -1):
        total = coef[k] + total * y
    powers = [torch.ones_like(x64)]
    for _ in range(l_max):
        powers.append(powers[-1] * x64)
    series = total * torch.stack(powers, -1) / torch.cumprod(2.0 * orders + 1.0, 0)
    xs = x64.clamp(min=1.0)
    rec = [torch.sin(xs) / xs]
    if l_max >= 1:
        rec.append((rec[0] - torch.cos(xs)) / xs)
    for l in range(1, l_max):
        rec.append((2 * l + 1) / xs * rec[l] - rec[l - 1])
    return torch.where(x64.unsqueeze(-1) < orders + 2.0, series, torch.stack(rec[:l_max + 1], -1)).to(x.dtype)


def spherical_bessel_zeros(l_max: int, n: int) -> np.ndarray:
    """The first ``n`` positive zeros of ``j_0 .. j_{l_max}`` (``(l_max + 1, n)``)."""
    zeros = np.zeros((l_max + 1, n + l_max))
    zeros[0] = np.arange(1, n + l_max + 1) * np.pi
    for l in range(1, l_max + 1):
        count = n + l_max - l
        lo = torch.tensor(zeros[l - 1, :count])
        hi = torch.tensor(zeros[l - 1, 1:count + 1])
        f_lo = spherical_bessel_jn(l, lo)[:, l]
        for _ in range(200):
            mid = 0.5 * (lo + hi)
            f_mid = spherical_bessel_jn(l, mid)[:, l]
            same = (f_mid > 0) == (f_lo > 0)
            lo, f_lo, hi = torch.where(same, mid, lo), torch.where(same, f_mid, f_lo), torch.where(same, hi, mid)
            if float((hi - lo).max()) <= 4.0 * np.finfo(np.float64).eps * float(hi.max()):
                break
        zeros[l, :count] = (0.5 * (lo + hi)).numpy()
    return zeros[:, :n]


def zonal_harmonics(l_max: int, cos_alpha: Tensor) -> Tensor:
    """``Y_l0 = sqrt((2l+1)/(4 pi)) P_l(cos alpha)`` for ``l = 0..l_max`` (Legendre recurrence)."""
    c = cos_alpha.to(torch.float64)
    p = [torch.ones_like(c), c]
    for l in range(1, l_max):
        p.append(((2 * l + 1) * c * p[l] - l * p[l - 1]) / (l + 1))
    out = [p[l] * math.sqrt((2 * l + 1) / (4.0 * math.pi)) for l in range(l_max + 1)]
    return torch.stack(out, -1).to(cos_alpha.dtype)


def real_spherical_harmonics(l_max: int, x: Tensor, y: Tensor, z: Tensor) -> Tensor:
    """Orthonormal real ``Y_lm`` of a unit vector, ``m = -l..l`` per ``l`` (associated Legendre
    recurrences in ``z``, ``cos(m phi)`` / ``sin(m phi)`` polynomials in ``x, y``)."""
    x64, y64, z64 = x.to(torch.float64), y.to(torch.float64), z.to(torch.float64)
    cm, sm = [torch.ones_like(z64)], [torch.zeros_like(z64)]
    for m in range(l_max):
        cm.append(cm[m] * x64 - sm[m] * y64)
        sm.append(sm[m] * x64 + cm[m] * y64)
    q = [[torch.zeros_like(z64) for _ in range(l + 1)] for l in range(l_max + 1)]
    dfact = 1.0
    for m in range(l_max + 1):
        if m > 0:
            dfact *= 2 * m - 1
        q[m][m] = torch.full_like(z64, dfact)
        if m + 1 <= l_max:
            q[m + 1][m] = (2 * m + 1) * z64 * q[m][m]
        for l in range(m + 2, l_max + 1):
            q[l][m] = ((2 * l - 1) * z64 * q[l - 1][m] - (l + m - 1) * q[l - 2][m]) / (l - m)
    out: List[Tensor] = []
    for l in range(l_max + 1):
        for m in range(-l, l + 1):
            a = abs(m)
            norm = math.sqrt((2 * l + 1) / (4.0 * math.pi) * math.factorial(l - a) / math.factorial(l + a))
            if m == 0:
                out.append(norm * q[l][0])
            elif m > 0:
                out.append(math.sqrt(2.0) * norm * q[l][a] * cm[a])
            else:
                out.append(math.sqrt(2.0) * norm * q[l][a] * sm[a])
    return torch.stack(out, -1).to(z.dtype)


class SphericalBesselBasis(nn.Module):
    def __init__(self, n_spherical: int = 7, n_radial: int = 6, cutoff: float = 5.0):
        super().__init__()
        self.n_spherical, self.n_radial, self.cutoff = n_spherical, n_radial, cutoff
        zeros = torch.tensor(spherical_bessel_zeros(n_spherical - 1, n_radial))
        j_next = torch.stack([spherical_bessel_jn(l + 1, zeros[l])[:, l + 1] for l in range(n_spherical)])
        norm = torch.sqrt(2.0 / (cutoff ** 3 * j_next ** 2))
        dt = torch.get_default_dtype()
        self.register_buffer("zeros", zeros.to(dt))
        self.register_buffer("norm", norm.to(dt))
        self.output_dim = n_spherical * n_radial

    def radial(self, r: Tensor) -> Tensor:
        """``(E, n_spherical, n_radial)``: ``norm_ln j_l(z_ln r / c)``."""
        x = (r.to(torch.float64) / self.cutoff)[:, None, None] * self.zeros.to(torch.float64)
        j = torch.stack([spherical_bessel_jn(l, x[:, l, :])[..., l] for l in range(self.n_spherical)], 1)
        return (self.norm.to(torch.float64) * j).to(r.dtype)

    def angular(self, cos_alpha: Tensor) -> Tensor:
        return zonal_harmonics(self.n_spherical - 1, cos_alpha)

    def forward(self, r: Tensor, cos_alpha: Tensor) -> Tensor:
        return (self.radial(r) * self.angular(cos_alpha)[:, :, None]).reshape(r.shape[0], self.output_dim)
