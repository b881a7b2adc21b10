"""Seeded synthetic structures of the benchmark shapes, with float64 Morse labels.

The labels are a Morse pair potential ``D [(1 - exp(-a (r - r0)))^2 - 1]`` with
``D = 0.2 eV``, ``a = 1.5 / A``, ``r0 = 1.4 A`` summed over pairs (over periodic
images within ``label_cutoff`` for cells), plus optional per-element reference
energies; forces and stress (virial / volume) come from float64 autograd. There is
no network here, so these stand in for the datasets of the reference's hub.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

MORSE_D, MORSE_A, MORSE_R0 = 0.2, 1.5, 1.4

#: config-2 elements {H, C, N, O, F, S, Cl} and their frequencies
ORGANIC_Z = [1, 6, 7, 8, 9, 16, 17]
ORGANIC_P = [0.50, 0.30, 0.08, 0.08, 0.02, 0.01, 0.01]


def _rejection_positions(rng: np.random.Generator, n: int, box: float, dmin: float,
                         max_tries: int = 20000) -> np.ndarray:
    pts = np.empty((n, 3))
    k = 0
    tries = 0
    while k < n:
        tries += 1
        if tries > max_tries * n:
            raise RuntimeError("could not place atoms with the requested minimum distance")
        p = rng.uniform(0.0, box, size=3)
        if k == 0 or np.min(np.sum((pts[:k] - p) ** 2, axis=1)) >= dmin * dmin:
            pts[k] = p
            k += 1
    return pts


def morse_labels(pos: torch.Tensor, z: torch.Tensor, cell: Optional[torch.Tensor] = None,
                 label_cutoff: float = 6.0, e0: Optional[Dict[int, float]] = None) -> Dict:
    """Float64 Morse energy, forces and (for cells) stress of one structure."""
    pos = pos.detach().to(torch.float64).clone().requires_grad_(True)
    n = pos.shape[0]
    strain = torch.zeros(3, 3, dtype=torch.float64, requires_grad=True)
    if cell is None:
        i, j = torch.triu_indices(n, n, 1)
        r = (pos[j] - pos[i]).norm(dim=-1)
        energy = (MORSE_D * ((1 - torch.exp(-MORSE_A * (r - MORSE_R0))) ** 2 - 1)).sum()
    else:
        from .neighborlist import build_neighbor_list
        c = cell.to(torch.float64)
        ei, sh = build_neighbor_list(pos.detach(), label_cutoff, c, torch.ones(3, dtype=torch.bool),
                                     engine="torch")
        sym = 0.5 * (strain + strain.T)
        p = pos + pos @ sym
        cc = c + c @ sym
        vec = p[ei[1]] - p[ei[0]] + sh.to(torch.float64) @ cc
        r = vec.norm(dim=-1)
        x = r / label_cutoff
        # smooth cosine taper so the periodic energy is continuous at the label cutoff
        taper = 0.5 * (torch.cos(math.pi * x) + 1.0)
        energy = 0.5 * (MORSE_D * ((1 - torch.exp(-MORSE_A * (r - MORSE_R0))) ** 2 - 1) * taper).sum()
    if e0:
        energy = energy + sum(e0.get(int(zz), 0.0) for zz in z.tolist())
    inputs = [pos] if cell is None else [pos, strain]
    grads = torch.autograd.grad(energy, inputs)
    out = {"energy": float(energy.detach()), "forces": (-grads[0]).detach()}
    if cell is not None:
        vol = float(torch.linalg.det(cell.to(torch.float64)).abs())
        out["stress"] = (grads[1] / vol).detach()
    return out


def organic_molecules(n_structures: int, seed: int = 0, n_min: int = 10, n_max: int = 60,
                      density: float = 0.1, dmin: float = 0.9, labels: bool = True,
                      e0_seed: int = 1) -> List[Dict]:
    """Config-2 molecules: 10-60 atoms of {H,C,N,O,F,S,Cl} in a cube at ``density`` atoms/A^3."""
    rng = np.random.default_rng(seed)
    e0rng = np.random.default_rng(e0_seed)
    e0 = {z: float(e0rng.normal()) for z in ORGANIC_Z}
    out = []
    for _ in range(n_structures):
        n = int(rng.integers(n_min, n_max + 1))
        box = (n / density) ** (1.0 / 3.0)
        pos = _rejection_positions(rng, n, box, dmin)
        z = rng.choice(ORGANIC_Z, size=n, p=ORGANIC_P)
        s = {"pos": torch.tensor(pos, dtype=torch.float64),
             "atomic_numbers": torch.tensor(z, dtype=torch.long)}
        if labels:
            s.update(morse_labels(s["pos"], s["atomic_numbers"], e0=e0))
        out.append(s)
    return out


def small_organic(n_structures: int = 250, seed: int = 0, labels: bool = True) -> List[Dict]:
    """Config-1 molecules: 21 atoms (8 H, 9 C, 4 O) in a 6 A cube, 0.9 A apart, jittered 0.05 A."""
    rng = np.random.default_rng(seed)
    z = np.array([1] * 8 + [6] * 9 + [8] * 4)
    out = []
    for _ in range(n_structures):
        pos = _rejection_positions(rng, 21, 6.0, 0.9) + rng.normal(0.0, 0.05, size=(21, 3))
        s = {"pos": torch.tensor(pos, dtype=torch.float64),
             "atomic_numbers": torch.tensor(rng.permutation(z), dtype=torch.long)}
        if labels:
            s.update(morse_labels(s["pos"], s["atomic_numbers"]))
        out.append(s)
    return out


def triclinic_crystals(n_structures: int, seed: int = 0, n_min: int = 8, n_max: int = 200,
                       dmin: float = 1.2, z_max: int = 89, labels: bool = True) -> List[Dict]:
    """Config-3 crystals: triclinic cells, 0.05-0.1 atoms/A^3, angles in 60-120 degrees."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_structures):
        n = int(rng.integers(n_min, n_max + 1))
        while True:
            ang = np.radians(rng.uniform(60.0, 120.0, size=3))
            ca, cb, cg = np.cos(ang)
            sg = np.sin(ang[2])
            v = 1 - ca * ca - cb * cb - cg * cg + 2 * ca * cb * cg
            if v > 0.05:
                break
        rho = rng.uniform(0.05, 0.1)
        ratio = rng.uniform(0.8, 1.25, size=3)
        # lengths a, b, c with the requested volume
        unit = np.sqrt(v) * ratio.prod()
        scale = (n / rho / unit) ** (1.0 / 3.0)
        a, b, c = ratio * scale
        cell = np.array([[a, 0, 0], [b * cg, b * sg, 0],
                         [c * cb, c * (ca - cb * cg) / sg, c * math.sqrt(v) / sg]])
        frac = np.empty((n, 3))
        k, tries = 0, 0
        imgs = np.array([[i, j, l] for i in (-1, 0, 1) for j in (-1, 0, 1) for l in (-1, 0, 1)])
        while k < n:
            tries += 1
            if tries > 200000:
                raise RuntimeError("crystal packing failed")
            f = rng.uniform(size=3)
            if k:
                d = (frac[:k, None, :] - f[None, None, :] + imgs[None]) @ cell
                if np.min(np.sum(d * d, axis=-1)) < dmin * dmin:
                    continue
            frac[k] = f
            k += 1
        pos = frac @ cell
        z = rng.integers(1, z_max + 1, size=n)
        s = {"pos": torch.tensor(pos, dtype=torch.float64), "atomic_numbers": torch.tensor(z),
             "cell": torch.tensor(cell, dtype=torch.float64), "pbc": torch.ones(3, dtype=torch.bool)}
        if labels:
            s.update(morse_labels(s["pos"], s["atomic_numbers"], s["cell"]))
        out.append(s)
    return out


def water_box(n_atoms: int, seed: int = 0, density: float = 0.1, oh: float = 0.96,
              angle_deg: float = 104.5, jitter: float = 0.1) -> Dict:
    """Config-4/5 water: ``n_atoms // 3`` H2O at random orientations on a jittered cubic lattice.

    The lattice spacing puts the box at ``density`` atoms per cubic Angstrom.
    """
    rng = np.random.default_rng(seed)
    n_mol = n_atoms // 3
    L = (3 * n_mol / density) ** (1.0 / 3.0)
    m = int(math.ceil(n_mol ** (1.0 / 3.0)))
    spacing = L / m
    idx = np.stack(np.meshgrid(np.arange(m), np.arange(m), np.arange(m), indexing="ij"), -1).reshape(-1, 3)
    idx = idx[rng.permutation(len(idx))[:n_mol]]
    centers = (idx + 0.5) * spacing + rng.uniform(-jitter, jitter, size=(n_mol, 3))
    half = math.radians(angle_deg) / 2
    local = np.array([[0.0, 0.0, 0.0], [oh * math.sin(half), oh * math.cos(half), 0.0],
                      [-oh * math.sin(half), oh * math.cos(half), 0.0]])
    # random rotations from unit quaternions
    q = rng.normal(size=(n_mol, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    R = np.stack([np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)], -1),
                  np.stack([2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)], -1),
                  np.stack([2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)], -1)], -2)
    pos = centers[:, None, :] + np.einsum("mij,kj->mki", R, local)
    pos = pos.reshape(-1, 3) % L
    z = np.tile(np.array([8, 1, 1]), n_mol)
    return {"pos": torch.tensor(pos, dtype=torch.float64), "atomic_numbers": torch.tensor(z),
            "cell": torch.eye(3, dtype=torch.float64) * L, "pbc": torch.ones(3, dtype=torch.bool)}
