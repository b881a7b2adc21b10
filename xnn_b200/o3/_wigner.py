"""Clebsch-Gordan (Wigner 3j) coupling tensors in the real spherical-harmonic basis.

The coupling tensor ``C[l1, l2, l3]`` of shape ``(2l1+1, 2l2+1, 2l3+1)`` is the unique
(up to sign) tensor invariant under ``D_l1 x D_l2 x D_l3``, normalised to unit
Frobenius norm. It is built from the complex (Condon-Shortley) coefficients of
Racah's closed formula, carried into the real basis by the standard unitary change
of basis with the ``(-i)^l`` phase that makes the result real. That is the
convention of e3nn's ``o3.wigner_3j``, which the reference builds its MACE ``U``
matrices and tensor-product paths from (``src/xnn/gnn/models/mace.py:68-146``).
The tests check invariance under rotations against the spherical harmonics of
:mod:`xnn_b200.o3._sh`.
"""
from __future__ import annotations

import functools
import math
from fractions import Fraction

import torch


def _fact(n: int) -> int:
    return math.factorial(n)


def _su2_cg(j1: int, m1: int, j2: int, m2: int, j3: int, m3: int) -> float:
    """<j1 m1 j2 m2 | j3 m3> from Racah's formula (exact rational arithmetic)."""
    if m3 != m1 + m2:
        return 0.0
    if not (abs(j1 - j2) <= j3 <= j1 + j2):
        return 0.0
    if abs(m1) > j1 or abs(m2) > j2 or abs(m3) > j3:
        return 0.0
    pre = Fraction((2 * j3 + 1) * _fact(j3 + j1 - j2) * _fact(j3 - j1 + j2) * _fact(j1 + j2 - j3),
                   _fact(j1 + j2 + j3 + 1))
    pre *= (_fact(j3 + m3) * _fact(j3 - m3) * _fact(j1 - m1) * _fact(j1 + m1)
            * _fact(j2 - m2) * _fact(j2 + m2))
    s = Fraction(0)
    kmin = max(0, j2 - j3 - m1, j1 - j3 + m2)
    kmax = min(j1 + j2 - j3, j1 - m1, j2 + m2)
    for k in range(kmin, kmax + 1):
        s += Fraction((-1) ** k, _fact(k) * _fact(j1 + j2 - j3 - k) * _fact(j1 - m1 - k)
                      * _fact(j2 + m2 - k) * _fact(j3 - j2 + m1 + k) * _fact(j3 - j1 - m2 + k))
    return float(s) * math.sqrt(float(pre))


def su2_clebsch_gordan(j1: int, j2: int, j3: int) -> torch.Tensor:
    """Complex-basis coefficients ``C[j1+m1, j2+m2, j3+m3]`` (float64)."""
    out = torch.zeros(2 * j1 + 1, 2 * j2 + 1, 2 * j3 + 1, dtype=torch.float64)
    for m1 in range(-j1, j1 + 1):
        for m2 in range(-j2, j2 + 1):
            m3 = m1 + m2
            if abs(m3) <= j3:
                out[j1 + m1, j2 + m2, j3 + m3] = _su2_cg(j1, m1, j2, m2, j3, m3)
    return out


def real_to_complex(l: int) -> torch.Tensor:
    """Unitary map between the complex and the real spherical-harmonic bases of degree ``l``.

    Row ``l+m`` of the result expresses complex index ``m``'s combination as in
    the standard real form (sine-like components for ``m < 0``, cosine-like for
    ``m > 0``), times the phase ``(-i)^l`` that makes the coupling tensors real.
    """
    q = torch.zeros(2 * l + 1, 2 * l + 1, dtype=torch.complex128)
    r2 = 1.0 / math.sqrt(2.0)
    for m in range(-l, 0):
        q[l + m, l + abs(m)] = r2
        q[l + m, l - abs(m)] = -1j * r2
    q[l, l] = 1.0
    for m in range(1, l + 1):
        q[l + m, l + abs(m)] = (-1) ** m * r2
        q[l + m, l - abs(m)] = 1j * (-1) ** m * r2
    return ((-1j) ** l) * q


@functools.lru_cache(maxsize=None)
def _wigner_3j_f64(l1: int, l2: int, l3: int) -> torch.Tensor:
    if not (abs(l1 - l2) <= l3 <= l1 + l2):
        raise ValueError(f"no coupling for ({l1}, {l2}, {l3})")
    q1, q2, q3 = real_to_complex(l1), real_to_complex(l2), real_to_complex(l3)
    c = su2_clebsch_gordan(l1, l2, l3).to(torch.complex128)
    c = torch.einsum("ij,kl,mn,ikn->jlm", q1, q2, torch.conj(q3.T), c)
    if c.imag.abs().max() > 1e-10:
        raise RuntimeError("coupling tensor is not real")
    c = c.real
    c = c / c.norm()
    c[c.abs() < 1e-15] = 0.0
    return c.contiguous()


def wigner_3j(l1: int, l2: int, l3: int, dtype=None, device=None) -> torch.Tensor:
    """The real coupling tensor ``(2l1+1, 2l2+1, 2l3+1)`` of unit Frobenius norm."""
    c = _wigner_3j_f64(int(l1), int(l2), int(l3))
    return c.to(dtype=dtype or torch.get_default_dtype(), device=device)
