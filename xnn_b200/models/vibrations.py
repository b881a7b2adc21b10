"""Second derivatives of a model's energy and harmonic vibrational analysis.

Behaviour follows the reference's ``src/xnn/common/models/vibrations.py`` (``hessian_vector_product``
at ``:108``, ``hessian`` at ``:146``, ``harmonic_analysis`` at ``:188``): Hessian-vector products by
differentiating the energy gradient once more (the fused MACE kernels are twice differentiable),
full Hessians per structure from ``3 n`` products, and harmonic frequencies / normal modes /
zero-point energy with translations and rotations projected out (``3 n - 5`` modes for a linear
molecule). Units: eV, Angstrom, u; wavenumbers in cm^-1.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
from torch import Tensor, nn

from ..data import elements
from ..data.atomic_graph import AtomicGraph

#: sqrt(eV / (A^2 u)) as a wavenumber in cm^-1, and h c in eV cm
WAVENUMBER = 521.4708382
HC = 1.239841984e-4


def _energy_gradient(model: nn.Module, data: AtomicGraph, create_graph: bool = False):
    pos = data.pos.detach().clone().requires_grad_(True)
    g = data.clone()
    g.pos = pos
    inner = getattr(model, "model", None)
    m = inner if inner is not None and hasattr(model, "compute_forces") else model
    energy = m(g)["energy"].sum()
    (grad,) = torch.autograd.grad(energy, pos, create_graph=True)
    return pos, grad


def hessian_vector_product(model: nn.Module, data: AtomicGraph, v: Tensor, create_graph: bool = False) -> Tensor:
    """``H v`` for ``v (N, 3)``: the directional derivative of the energy gradient."""
    pos, grad = _energy_gradient(model, data)
    (hv,) = torch.autograd.grad((grad * v).sum(), pos, create_graph=create_graph)
    return hv


def hessian(model: nn.Module, data: AtomicGraph, create_graph: bool = False) -> List[Tensor]:
    """The Hessian ``(3 n_b, 3 n_b)`` of every structure of the batch (eV / A^2)."""
    pos, grad = _energy_gradient(model, data)
    flat = grad.reshape(-1)
    n = pos.shape[0]
    rows = []
    for k in range(3 * n):
        (h,) = torch.autograd.grad(flat[k], pos, retain_graph=True, create_graph=create_graph)
        rows.append(h.reshape(-1))
    H = torch.stack(rows)
    out = []
    for b in range(data.num_graphs):
        idx = torch.nonzero(data.batch == b).flatten()
        cols = (3 * idx[:, None] + torch.arange(3, device=idx.device)).reshape(-1)
        out.append(H[cols][:, cols])
    return out


def harmonic_analysis(hessian: Tensor, positions: Tensor, masses: Optional[Tensor] = None,
                      atomic_numbers: Optional[Tensor] = None, linear_tolerance: float = 1e-5) -> Dict[str, object]:
    """Frequencies (cm^-1, ascending, imaginary as negative), normal modes, Cartesian
    displacements, zero-point energy (eV) and the (projected) mass-weighted Hessians of one
    structure; differentiable with respect to ``hessian``."""
    dtype, device = hessian.dtype, hessian.device
    if masses is None:
        if atomic_numbers is None:
            raise ValueError("harmonic_analysis needs masses or atomic_numbers")
        masses = elements.masses(atomic_numbers.to(device), dtype)
    m = masses.to(dtype=dtype, device=device)
    x = positions.detach().to(dtype=dtype, device=device)
    n = x.shape[0]
    s = m.sqrt().repeat_interleave(3)
    Hmw = 0.5 * (hessian + hessian.transpose(0, 1)) / (s[:, None] * s[None, :])
    r = x - (m[:, None] * x).sum(0) / m.sum()
    eye = torch.eye(3, dtype=dtype, device=device)
    inertia = (m * (r * r).sum(1)).sum() * eye - torch.einsum("i,ij,ik->jk", m, r, r)
    moments = torch.linalg.eigvalsh(inertia)
    linear = n == 2 or (n > 2 and bool(moments[0] <= linear_tolerance * moments[2]))
    n_ext = 3 if n == 1 else (5 if linear else 6)
    sm = m.sqrt()[:, None]
    ext = [(sm * eye[k]).reshape(-1) for k in range(3)]
    ext += [(sm * torch.linalg.cross(eye[k].expand_as(r), r)).reshape(-1) for k in range(3)]
    U, _, _ = torch.linalg.svd(torch.stack(ext, 1), full_matrices=True)
    E, B = U[:, :n_ext], U[:, n_ext:]
    K = B.t() @ Hmw @ B
    lam, Y = torch.linalg.eigh(K) if K.shape[0] else (K.new_zeros(0), K)
    modes = (B @ Y).t().reshape(-1, n, 3)
    freq = torch.sign(lam) * lam.abs().sqrt() * WAVENUMBER
    P = torch.eye(3 * n, dtype=dtype, device=device) - E @ E.t()
    return {"frequencies": freq, "eigenvalues": lam, "modes": modes, "displacements": modes / m.sqrt()[None, :, None],
            "zero_point_energy": 0.5 * HC * freq.clamp(min=0.0).sum(), "mass_weighted_hessian": Hmw,
            "projected_hessian": P @ Hmw @ P, "linear": linear}
