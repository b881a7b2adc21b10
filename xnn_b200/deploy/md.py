"""Molecular dynamics drivers over :class:`~xnn_b200.parallel.domain.DomainParallel`.

Units: positions in Angstrom, time in fs, energies in eV, masses in amu. Every process
integrates the atoms it owns; when the plan no longer holds (atoms moved more than the skin
allows) the atoms are handed to their new owners (``DomainParallel.reshard``). With one
process the same code runs the whole structure, keeping the box's own periodicity.

The reference has no standalone integrator for ML potentials (its MD lives in ASE, LAMMPS
and its ``StepGraph``); this is the velocity-Verlet loop of the large-system MD benchmark.
"""
from __future__ import annotations

from typing import Callable, Dict, Optional

import torch
import torch.distributed as dist
from torch import Tensor

from ..data import elements
from ..data.atomic_graph import AtomicGraph
from ..parallel.domain import DomainParallel

#: acceleration of 1 eV/Angstrom on 1 amu, in Angstrom/fs^2
ACC_UNIT = 9.648533212e-3
#: Boltzmann constant in eV/K
KB_EV = 8.617333262e-5


def maxwell_boltzmann(masses: Tensor, temperature_k: float, seed: int = 0) -> Tensor:
    """Velocities (Angstrom/fs) drawn at ``temperature_k`` with zero total momentum; the same
    for every process (drawn on the CPU for the whole structure)."""
    g = torch.Generator().manual_seed(seed)
    m = masses.detach().to("cpu", torch.float64)
    sigma = torch.sqrt(KB_EV * temperature_k * ACC_UNIT / m)[:, None]
    v = torch.randn(m.shape[0], 3, generator=g, dtype=torch.float64) * sigma
    if m.shape[0] > 1:
        v -= (m[:, None] * v).sum(0) / m.sum()
    return v.to(masses.device)


class VelocityVerlet:
    """NVE velocity Verlet for a structure split over the processes (or whole on one).

    ``potential`` is a :class:`DomainParallel` or a model (wrapped with ``skin``). Collective:
    every process constructs it and calls :meth:`step` together.
    """

    def __init__(self, potential, graph: AtomicGraph, dt_fs: float = 0.5, temperature_k: float = 0.0,
                 seed: int = 0, masses: Optional[Tensor] = None, velocities: Optional[Tensor] = None,
                 skin: float = 1.0):
        self.dp = potential if isinstance(potential, DomainParallel) else DomainParallel(potential, skin=skin)
        self.dt = float(dt_fs)
        periodic = graph.cell is not None and graph.pbc is not None and bool(graph.pbc.any())
        self.cell = graph.cell[0] if periodic else None
        self.plan = self.dp.plan(graph)
        m_all = masses if masses is not None else elements.masses(graph.atomic_numbers)
        m_all = m_all.to(graph.pos.device, torch.float64)
        v_all = velocities if velocities is not None else maxwell_boltzmann(m_all, temperature_k, seed)
        owned = self.plan.owned
        self.pos = graph.pos.detach()[owned].clone()
        self.vel = v_all.to(self.pos.device, self.pos.dtype)[owned].clone()
        self.mass = m_all[owned].to(self.pos.dtype)
        self.rebuilds = 0
        self.n_steps = 0
        out = self.dp.evaluate(self.plan, self.pos, self.cell)
        self.forces, self.energy = out["forces"].detach(), out["energy"].detach()

    def _acc(self) -> Tensor:
        return self.forces * (ACC_UNIT / self.mass)[:, None]

    def kinetic_energy(self) -> Tensor:
        ke = (0.5 / ACC_UNIT) * (self.mass[:, None] * self.vel * self.vel).sum().to(torch.float64).reshape(1)
        if self.plan.world > 1:
            dist.all_reduce(ke, group=self.dp.group)
        return ke

    def step(self) -> Dict[str, float]:
        """One step; returns the potential, kinetic and total energy after it (eV)."""
        dt = self.dt
        self.vel = self.vel + (0.5 * dt) * self._acc()
        self.pos = self.pos + dt * self.vel
        if not self.dp.holds(self.plan, self.pos, self.cell):
            self.plan, self.pos, self.vel, self.mass = self.dp.reshard(self.plan, self.pos, self.vel, self.mass,
                                                                      cell=self.cell)
            self.rebuilds += 1
        out = self.dp.evaluate(self.plan, self.pos, self.cell)
        self.forces, self.energy = out["forces"].detach(), out["energy"].detach()
        self.vel = self.vel + (0.5 * dt) * self._acc()
        self.n_steps += 1
        ke = float(self.kinetic_energy())
        pe = float(self.energy)
        return {"potential": pe, "kinetic": ke, "total": pe + ke}

    def run(self, n_steps: int, callback: Optional[Callable[[int, Dict[str, float]], None]] = None):
        log = None
        for i in range(n_steps):
            log = self.step()
            if callback is not None:
                callback(i, log)
        return log

    def gather_positions(self) -> Tensor:
        """Positions of every atom of the structure, in its atom order (collective)."""
        return self.dp._gather(self.plan, self.pos)
