"""Functions on the sphere sampled on a ``(beta, alpha)`` grid and their real spherical-harmonic
coefficients, with e3nn's ``ToS2Grid`` / ``FromS2Grid`` conventions (the reference's EquiformerV2
builds its grid activations on them, ``src/xnn/trfnn/models/equiformer_v2.py:100``).

Grid: ``beta_i = (i + 1/2) pi / res_beta`` measured from the y axis, ``alpha_j = 2 pi j / res_alpha``
in the z-x plane, the point ``(sin b sin a, cos b, sin b cos a)``. A harmonic of order ``m``
separates into a function of beta (``shb``, ``(2 lmax + 1, res_beta, (lmax + 1)^2)``, nonzero only
in row ``m + lmax``) times ``sqrt(2) sin(|m| a)`` (``m < 0``), ``1`` or ``sqrt(2) cos(m a)``
(``sha``, ``(res_alpha, 2 lmax + 1)``). The beta factors are obtained here by sampling each harmonic
on ``2 lmax + 1`` equispaced azimuths and projecting onto its order's azimuthal factor (exact: the
products are trigonometric polynomials of degree at most ``2 lmax``). Analysis integrates with the
Driscoll-Healy weights in beta (Driscoll and Healy, Adv. Appl. Math. 15, 1994).
"""
from __future__ import annotations

import math
from functools import lru_cache
from typing import Optional, Tuple

import torch
from torch import Tensor, nn

from ._sh import spherical_harmonics


def s2_grid(res_beta: int, res_alpha: int, dtype=torch.float64) -> Tuple[Tensor, Tensor]:
    betas = (torch.arange(res_beta, dtype=dtype) + 0.5) / res_beta * math.pi
    alphas = torch.arange(res_alpha, dtype=dtype) / res_alpha * (2.0 * math.pi)
    return betas, alphas


def spherical_harmonics_alpha(lmax: int, alpha: Tensor) -> Tensor:
    """``(..., 2 lmax + 1)`` azimuthal factors of orders ``-lmax .. lmax``."""
    a = alpha.unsqueeze(-1)
    up = torch.arange(1, lmax + 1, dtype=alpha.dtype, device=alpha.device)
    return torch.cat([math.sqrt(2.0) * torch.sin(up.flip(0) * a), torch.ones_like(a),
                      math.sqrt(2.0) * torch.cos(up * a)], -1)


def grid_points(betas: Tensor, alphas: Tensor) -> Tensor:
    b, a = torch.meshgrid(betas, alphas, indexing="ij")
    return torch.stack([torch.sin(b) * torch.sin(a), torch.cos(b), torch.sin(b) * torch.cos(a)], -1)


@lru_cache(maxsize=None)
def _beta_factors(lmax: int, res_beta: int) -> Tensor:
    """``shb`` of the integral-normalised harmonics, float64."""
    betas, _ = s2_grid(res_beta, 1)
    n_alpha = 2 * lmax + 1
    alphas = torch.arange(n_alpha, dtype=torch.float64) / n_alpha * (2.0 * math.pi)
    y = spherical_harmonics(list(range(lmax + 1)), grid_points(betas, alphas), normalize=True,
                            normalization="integral")                               # (B, A, I)
    coef = torch.einsum("bai,am->mbi", y, spherical_harmonics_alpha(lmax, alphas)) / n_alpha
    order = torch.tensor([m for l in range(lmax + 1) for m in range(-l, l + 1)]) + lmax
    keep = torch.arange(2 * lmax + 1)[:, None] == order[None, :]
    return coef * keep[:, None, :]


@lru_cache(maxsize=None)
def quadrature_weights(b: int) -> Tensor:
    """Driscoll-Healy weights of the ``2b`` beta samples, normalised to ``1 / (2b)^2`` in total."""
    beta = (torch.arange(2 * b, dtype=torch.float64) + 0.5) * math.pi / (2 * b)
    k = torch.arange(b, dtype=torch.float64)
    series = (torch.sin((2 * k + 1)[None] * beta[:, None]) / (2 * k + 1)[None]).sum(1)
    return (2.0 / b) * torch.sin(beta) * series / (2.0 * (2 * b) ** 2)


def _degrees(lmax: int) -> Tensor:
    return torch.tensor([l for l in range(lmax + 1) for _ in range(2 * l + 1)], dtype=torch.float64)


def _resolution(lmax: int, res) -> Tuple[int, int]:
    if res is None:
        return 2 * (lmax + 1), 2 * (lmax + 1)
    return int(res[0]), int(res[1])


class ToS2Grid(nn.Module):
    """Coefficients ``(..., (lmax + 1)^2)`` to grid values ``(..., res_beta, res_alpha)``.
    ``normalization`` scales degree ``l`` so that a unit coefficient vector gives a unit mean
    square (``component``), a unit-norm harmonic per degree (``norm``) or the plain integral-
    normalised harmonic (``integral``)."""

    def __init__(self, lmax: int, res: Optional[Tuple[int, int]] = None, normalization: str = "component",
                 dtype=None, device=None):
        super().__init__()
        self.lmax = int(lmax)
        self.res_beta, self.res_alpha = _resolution(self.lmax, res)
        l = _degrees(self.lmax)
        if normalization == "component":
            n = math.sqrt(4 * math.pi) / torch.sqrt(2 * l + 1) / math.sqrt(self.lmax + 1)
        elif normalization == "norm":
            n = math.sqrt(4 * math.pi) * torch.ones_like(l) / math.sqrt(self.lmax + 1)
        elif normalization == "integral":
            n = torch.ones_like(l)
        else:
            raise ValueError(f"unknown normalization {normalization!r}")
        dtype = dtype or torch.get_default_dtype()
        _, alphas = s2_grid(self.res_beta, self.res_alpha)
        self.register_buffer("shb", (_beta_factors(self.lmax, self.res_beta) * n).to(dtype=dtype, device=device))
        self.register_buffer("sha", spherical_harmonics_alpha(self.lmax, alphas).to(dtype=dtype, device=device))

    def forward(self, x: Tensor) -> Tensor:
        y = torch.einsum("mbi,...i->...bm", self.shb, x)
        return torch.einsum("am,...bm->...ba", self.sha, y)


class FromS2Grid(nn.Module):
    """Grid values ``(..., res_beta, res_alpha)`` to coefficients ``(..., (lmax + 1)^2)`` by
    quadrature (``res_beta`` even); the inverse of :class:`ToS2Grid` of the same normalisation on
    band-limited functions."""

    def __init__(self, res: Optional[Tuple[int, int]] = None, lmax: Optional[int] = None,
                 normalization: str = "component", lmax_in: Optional[int] = None, dtype=None, device=None):
        super().__init__()
        if lmax is None:
            raise ValueError("lmax is required")
        self.lmax = int(lmax)
        self.res_beta, self.res_alpha = _resolution(self.lmax, res)
        if self.res_beta % 2:
            raise ValueError(f"the quadrature needs an even beta resolution, got {self.res_beta}")
        l = _degrees(self.lmax)
        if normalization == "component":
            n = math.sqrt(4 * math.pi) * torch.sqrt(2 * l + 1) * math.sqrt(self.lmax + 1)
        elif normalization == "norm":
            n = math.sqrt(4 * math.pi) * torch.ones_like(l) * math.sqrt(self.lmax + 1)
        elif normalization == "integral":
            n = 4 * math.pi * torch.ones_like(l)
        else:
            raise ValueError(f"unknown normalization {normalization!r}")
        qw = quadrature_weights(self.res_beta // 2) * self.res_beta ** 2 / self.res_alpha
        dtype = dtype or torch.get_default_dtype()
        _, alphas = s2_grid(self.res_beta, self.res_alpha)
        shb = _beta_factors(self.lmax, self.res_beta) * n * qw[None, :, None]
        self.register_buffer("shb", shb.to(dtype=dtype, device=device))
        self.register_buffer("sha", spherical_harmonics_alpha(self.lmax, alphas).to(dtype=dtype, device=device))

    def forward(self, x: Tensor) -> Tensor:
        y = torch.einsum("am,...ba->...bm", self.sha, x)
        return torch.einsum("mbi,...bm->...i", self.shb, y)
