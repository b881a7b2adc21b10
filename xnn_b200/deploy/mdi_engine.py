"""MolSSI Driver Interface (MDI) engine.

The command set follows the reference's engine (``src/xnn/common/deploy/mdi_engine.py:78-620``):
``>NATOMS``, ``>ELEMENTS``, ``>CELL``, ``>COORDS`` (driver to engine) and ``<NATOMS``,
``<ENERGY``, ``<FORCES``, ``<STRESS``, ``<COORDS`` (engine to driver), ``EXIT``; MDI's atomic
units on the wire (bohr, hartree, hartree/bohr). The transport is a small object with
``recv_command()``, ``recv(count, dtype)`` and ``send(values, dtype)``; :func:`mdi_comm` adapts
the ``mdi`` Python package when it is installed (TCP or MPI), and tests drive the engine
through an in-memory one.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from ..data.dataset import structure_to_graph
from ..models.dispersion import BOHR, HARTREE


class MDIEngine:
    def __init__(self, potential, device: str = "cpu", cutoff: Optional[float] = None):
        from ..models.outputs import ForceStressOutput
        if not hasattr(potential, "compute_forces"):
            potential = ForceStressOutput(potential, compute_stress=True)
        self.model = potential.to(device).eval()
        self.device = device
        self.cutoff = float(cutoff if cutoff is not None else self.model.cutoff)
        self.natoms = 0
        self.elements: Optional[np.ndarray] = None
        self.coords: Optional[np.ndarray] = None     # Angstrom
        self.cell: Optional[np.ndarray] = None       # Angstrom, rows
        self._result = None

    def _evaluate(self):
        if self._result is None:
            s = {"pos": torch.as_tensor(self.coords, dtype=torch.float64),
                 "atomic_numbers": torch.as_tensor(self.elements, dtype=torch.long)}
            if self.cell is not None and np.abs(self.cell).sum() > 0:
                s["cell"] = torch.as_tensor(self.cell, dtype=torch.float64)
                s["pbc"] = np.ones(3, dtype=bool)
            g = structure_to_graph(s, self.cutoff, device=self.device)
            out = self.model(g)
            self._result = {k: v.detach().cpu().to(torch.float64).numpy() for k, v in out.items()
                            if torch.is_tensor(v)}
        return self._result

    def handle(self, command: str, comm) -> bool:
        """Execute one command; False after ``EXIT``."""
        c = command.strip()
        if c == "EXIT":
            return False
        if c == ">NATOMS":
            self.natoms = int(comm.recv(1, "int")[0])
        elif c == "<NATOMS":
            comm.send([self.natoms], "int")
        elif c == ">ELEMENTS":
            self.elements = np.asarray(comm.recv(self.natoms, "int"), dtype=np.int64)
        elif c == ">CELL":
            self.cell = np.asarray(comm.recv(9, "double"), dtype=np.float64).reshape(3, 3) * BOHR
        elif c == ">COORDS":
            self.coords = np.asarray(comm.recv(3 * self.natoms, "double"), dtype=np.float64).reshape(-1, 3) * BOHR
        elif c == "<COORDS":
            comm.send((self.coords / BOHR).reshape(-1).tolist(), "double")
        elif c == "<ENERGY":
            comm.send([float(self._evaluate()["energy"].sum()) / HARTREE], "double")
        elif c == "<FORCES":
            comm.send((self._evaluate()["forces"] * (BOHR / HARTREE)).reshape(-1).tolist(), "double")
        elif c == "<STRESS":
            st = self._evaluate().get("stress")
            st = np.zeros(9) if st is None else st.reshape(-1)
            comm.send((st * (BOHR ** 3 / HARTREE)).tolist(), "double")
        else:
            raise ValueError(f"unsupported MDI command {c!r}")
        if c.startswith(">"):
            self._result = None
        return True

    def serve(self, comm) -> None:
        while self.handle(comm.recv_command(), comm):
            pass


def mdi_comm(options: str):  # pragma: no cover - needs the mdi package and a driver
    """An MDI transport over the ``mdi`` package (``-role ENGINE -name xnn -method TCP ...``)."""
    import mdi
    mdi.MDI_Init(options)
    c = mdi.MDI_Accept_Communicator()
    kinds = {"int": mdi.MDI_INT, "double": mdi.MDI_DOUBLE}

    class _Comm:
        def recv_command(self):
            return mdi.MDI_Recv_Command(c)

        def recv(self, count, kind):
            return mdi.MDI_Recv(count, kinds[kind], c)

        def send(self, values, kind):
            mdi.MDI_Send(values, len(values), kinds[kind], c)

    return _Comm()
