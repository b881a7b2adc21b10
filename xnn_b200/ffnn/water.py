"""Config-5 test system: a water box with random permanent multipoles and polarizabilities."""
from __future__ import annotations

import torch

from ..data import synthetic


def multipole_water(n_atoms: int = 100_000, seed: int = 0, device="cpu", dtype=torch.float64):
    """Positions (A), cell, charges / dipoles / traceless quadrupoles ~ N(0, 0.3 e A^k) and
    polarizabilities uniform in 0.8-1.4 A^3; molecules are consecutive O, H, H triples.

    The box keeps water's 0.1 atoms/A^3 (a 100,000-atom box is 100.4 A wide)."""
    s = synthetic.water_box(n_atoms, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    n = s["pos"].shape[0]
    q = 0.3 * torch.randn(n, generator=g, dtype=torch.float64)
    d = 0.3 * torch.randn(n, 3, generator=g, dtype=torch.float64)
    A = 0.3 * torch.randn(n, 3, 3, generator=g, dtype=torch.float64)
    A = 0.5 * (A + A.transpose(1, 2))
    Q = A - torch.eye(3, dtype=torch.float64) * (A.diagonal(dim1=1, dim2=2).sum(-1) / 3.0)[:, None, None]
    pol = 0.8 + 0.6 * torch.rand(n, generator=g, dtype=torch.float64)
    mol = torch.arange(n) // 3
    to = lambda t: t.to(device=device, dtype=dtype) if t.is_floating_point() else t.to(device)  # noqa: E731
    return {"pos": to(s["pos"]), "cell": to(s["cell"]), "q": to(q), "d": to(d), "Q": to(Q), "pol": to(pol),
            "molecule": mol.to(device)}
