"""Radial bases (``src/xnn/common/featurizers/radial.py``)."""
from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor, nn


class GaussianRBF(nn.Module):
    """``exp(-gamma (r - mu_k)^2)`` with ``n_rbf`` centres evenly spaced on ``[start, cutoff]``."""

    def __init__(self, n_rbf: int = 50, cutoff: float = 5.0, start: float = 0.0,
                 gamma: Optional[float] = None, trainable: bool = False, endpoint: bool = True):
        super().__init__()
        centers = torch.linspace(start, cutoff, n_rbf) if endpoint else torch.linspace(start, cutoff, n_rbf + 1)[:n_rbf]
        width = float(centers[1] - centers[0]) if n_rbf > 1 else 1.0
        g = float(gamma) if gamma is not None else 0.5 / width ** 2
        if trainable:
            self.centers, self.gamma = nn.Parameter(centers), nn.Parameter(torch.tensor(g))
        else:
            # a plain float (the state dict holds only the centres, as the reference's)
            self.register_buffer("centers", centers)
            self.gamma = g

    def forward(self, r: Tensor) -> Tensor:
        return torch.exp(-self.gamma * (r[..., None] - self.centers) ** 2)


class ExpNormalSmearing(nn.Module):
    """TorchMD-Net basis ``cos-cutoff(r) exp(-beta (exp(alpha (start - r)) - mu)^2)``."""

    def __init__(self, n_rbf: int = 32, cutoff: float = 5.0, start: float = 0.0,
                 trainable: bool = True):
        super().__init__()
        self.cutoff, self.start, self.n_rbf = float(cutoff), float(start), n_rbf
        self.alpha = 5.0 / (cutoff - start)
        means, betas = self._initial(torch.get_default_dtype())
        if trainable:
            self.means, self.betas = nn.Parameter(means), nn.Parameter(betas)
        else:
            self.register_buffer("means", means)
            self.register_buffer("betas", betas)

    def _initial(self, dtype):
        s = math.exp(-self.cutoff + self.start)
        means = torch.linspace(s, 1.0, self.n_rbf, dtype=dtype)
        betas = torch.full((self.n_rbf,), (2.0 / self.n_rbf * (1.0 - s)) ** -2, dtype=dtype)
        return means, betas

    def forward(self, r: Tensor) -> Tensor:
        r = r[..., None]
        env = 0.5 * (torch.cos(math.pi * r / self.cutoff) + 1.0) * (r < self.cutoff)
        return env * torch.exp(-self.betas * (torch.exp(self.alpha * (self.start - r)) - self.means) ** 2)


class BesselRBF(nn.Module):
    """``prefactor sin(n pi r / rc) / r`` for ``n = 1..n_rbf``; prefactor ``sqrt(2/rc)`` by default."""

    def __init__(self, n_rbf: int = 8, cutoff: float = 5.0, trainable: bool = False,
                 prefactor: Optional[float] = None):
        super().__init__()
        self.cutoff = float(cutoff)
        freqs = math.pi * torch.arange(1, n_rbf + 1, dtype=torch.get_default_dtype())
        if trainable:
            self.freqs = nn.Parameter(freqs)
        else:
            self.register_buffer("freqs", freqs)
        self.norm = math.sqrt(2.0 / cutoff) if prefactor is None else float(prefactor)

    def forward(self, r: Tensor) -> Tensor:
        r = r.clamp(min=1e-8)[..., None]
        return self.norm * torch.sin(self.freqs * r / self.cutoff) / r


class SmoothBesselRBF(nn.Module):
    """Orthogonal combinations of spherical Bessel functions vanishing smoothly at ``rc`` (Kocer)."""

    def __init__(self, n_rbf: int = 3, cutoff: float = 5.0):
        super().__init__()
        self.cutoff = float(cutoff)
        n = n_rbf
        e = torch.zeros(n, dtype=torch.float64)
        d = torch.zeros(n, dtype=torch.float64)
        for k in range(n):
            e[k] = k ** 2 * (k + 2) ** 2 / (4 * (k + 1) ** 4 + 1)
        d[0] = 1.0
        for k in range(1, n):
            d[k] = 1.0 - e[k] / d[k - 1]
        self.register_buffer("e", e.to(torch.get_default_dtype()))
        self.register_buffer("d", d.to(torch.get_default_dtype()))

    def forward(self, r: Tensor) -> Tensor:
        rc = self.cutoff
        n = self.e.shape[0]
        r = r[..., None]
        k = torch.arange(n, device=r.device, dtype=r.dtype)
        a = (-1) ** k * math.sqrt(2.0) * math.pi / rc ** 1.5 * (k + 1) * (k + 2) / torch.sqrt((k + 1) ** 2 + (k + 2) ** 2)
        x1 = r * (k + 1) * math.pi / rc
        x2 = r * (k + 2) * math.pi / rc
        f = a * (torch.sinc(x1 / math.pi) + torch.sinc(x2 / math.pi))
        out = [f[..., 0]]
        prev = f[..., 0]
        for m in range(1, n):
            g = (f[..., m] + torch.sqrt(self.e[m] / self.d[m - 1]) * prev) / torch.sqrt(self.d[m])
            out.append(g)
            prev = g
        return torch.stack(out, -1) * (r < rc)


RADIAL_BASES = ("gaussian", "bessel", "expnorm", "smooth_bessel")


def make_radial_basis(name: str, n_rbf: int, cutoff: float, trainable: bool = False, *,
                      gamma: Optional[float] = None, prefactor: Optional[float] = None) -> nn.Module:
    if name == "gaussian":
        return GaussianRBF(n_rbf, cutoff, gamma=gamma, trainable=trainable)
    if name == "bessel":
        return BesselRBF(n_rbf, cutoff, trainable=trainable, prefactor=prefactor)
    if name == "expnorm":
        return ExpNormalSmearing(n_rbf, cutoff, trainable=trainable)
    if name == "smooth_bessel":
        return SmoothBesselRBF(n_rbf, cutoff)
    raise ValueError(f"unknown radial basis {name!r}; options: {RADIAL_BASES}")


class ExponentialBernsteinRBF(nn.Module):
    """Bernstein polynomials of ``x = exp(-gamma r)``: ``C(n-1, k) x^k (1 - x)^(n-1-k)`` (SpookyNet),
    evaluated in log space; ``gamma = softplus(gamma_raw)`` (trainable by default)."""

    def __init__(self, n_rbf: int = 16, gamma: float = 0.5 / 0.5291772109044924, trainable: bool = True,
                 exp_weighting: bool = False):
        super().__init__()
        self.n_rbf, self.exp_weighting = int(n_rbf), bool(exp_weighting)
        k = torch.arange(self.n_rbf, dtype=torch.float64)
        n = float(self.n_rbf - 1)
        log_binom = math.lgamma(n + 1.0) - torch.lgamma(k + 1.0) - torch.lgamma(n - k + 1.0)
        dt = torch.get_default_dtype()
        self.register_buffer("log_binom", log_binom.to(dt), persistent=False)
        self.register_buffer("power_x", k.to(dt), persistent=False)
        self.register_buffer("power_1mx", (n - k).to(dt), persistent=False)
        raw = torch.tensor(float(gamma) + math.log(-math.expm1(-float(gamma))), dtype=dt)   # softplus^-1
        if trainable:
            self.gamma_raw = nn.Parameter(raw)
        else:
            self.register_buffer("gamma_raw", raw)

    @property
    def gamma(self) -> Tensor:
        return nn.functional.softplus(self.gamma_raw)

    def forward(self, r: Tensor) -> Tensor:
        log_x = -nn.functional.softplus(self.gamma_raw) * r.unsqueeze(-1)
        rbf = torch.exp(self.log_binom + self.power_x * log_x + self.power_1mx * torch.log(-torch.expm1(log_x)))
        return rbf * torch.exp(log_x) if self.exp_weighting else rbf
