"""MolSSI Driver Interface (MDI) engine.

The command set follows the reference's engine (``src/xnn/common/deploy/mdi_engine.py:78-620``):
``>NATOMS``, ``>ELEMENTS``, ``>CELL``, ``>COORDS``, ``>TOTCHARGE`` (driver to engine) and
``<NATOMS``, ``<ENERGY``, ``<FORCES``, ``<STRESS``, ``<COORDS``, ``<CELL`` (engine to driver),
``SCF`` (evaluate now) and ``EXIT``; MDI's atomic units on the wire (bohr, hartree,
hartree/bohr, hartree/bohr^3; the stress with the pressure sign, as MDI drivers expect). The
model is evaluated lazily, once per new geometry: positions and cell in float64, the model in
its own dtype, the graph built on the model's device; every 100 evaluations the time split
(graph / model / read-back) and the atom-step rate are logged, and :meth:`MDIEngine.stats`
returns them. The transport is a small object with ``recv_command()``, ``recv(count, dtype)`` and
``send(values, dtype)``; :func:`mdi_comm` adapts the ``mdi`` Python package when it is installed
(TCP or MPI), and tests drive the engine through an in-memory one.
"""
from __future__ import annotations

import logging
import time
from typing import Dict, Optional

import numpy as np
import torch

from ..data.dataset import structure_to_graph
from ..models.dispersion import BOHR, HARTREE


log = logging.getLogger(__name__)


class MDIEngine:
    def __init__(self, potential, device: str = "cpu", cutoff: Optional[float] = None, total_charge: float = 0.0):
        from ..models.outputs import ForceStressOutput
        if not hasattr(potential, "compute_forces"):
            potential = ForceStressOutput(potential, compute_stress=True)
        self.model = potential.to(device).eval()
        for p in self.model.parameters():
            p.requires_grad_(False)
        self.device = torch.device(device)
        self.dtype = next(self.model.parameters()).dtype
        self.cutoff = float(cutoff if cutoff is not None else self.model.cutoff)
        self.total_charge = float(total_charge)
        self.natoms = 0
        self.elements: Optional[np.ndarray] = None
        self.coords: Optional[np.ndarray] = None     # Angstrom
        self.cell: Optional[np.ndarray] = None       # Angstrom, rows
        self._result = None
        self._n, self._t = 0, {"graph": 0.0, "model": 0.0, "read": 0.0, "total": 0.0}

    @classmethod
    def from_pretrained(cls, source, device: str = "cpu", **kw) -> "MDIEngine":
        """An engine for a checkpoint path, registered name, URL or DOI (see :mod:`xnn_b200.hub`)."""
        from ..hub import from_pretrained
        return cls(from_pretrained(source), device=device, **kw)

    def _sync(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def _evaluate(self):
        if self._result is None:
            if self.coords is None or self.elements is None:
                raise RuntimeError("no >ELEMENTS / >COORDS received before a result was requested")
            t0 = time.perf_counter()
            s = {"pos": torch.as_tensor(self.coords, dtype=torch.float64),
                 "atomic_numbers": torch.as_tensor(self.elements, dtype=torch.long),
                 "total_charge": self.total_charge}
            if self.cell is not None and np.abs(self.cell).sum() > 0:
                s["cell"] = torch.as_tensor(self.cell, dtype=torch.float64)
                s["pbc"] = np.ones(3, dtype=bool)
            g = structure_to_graph(s, self.cutoff, device=self.device)
            g.compute_dtype = self.dtype
            self._sync()
            t1 = time.perf_counter()
            out = self.model(g)
            self._sync()
            t2 = time.perf_counter()
            self._result = {k: v.detach().cpu().to(torch.float64).numpy() for k, v in out.items()
                            if torch.is_tensor(v)}
            t3 = time.perf_counter()
            self._n += 1
            for k, dt in (("graph", t1 - t0), ("model", t2 - t1), ("read", t3 - t2), ("total", t3 - t0)):
                self._t[k] += dt
            if self._n % 100 == 0:
                st = self.stats()
                log.info("evaluation %d: graph %.2f, model %.2f, read-back %.2f ms; %.1f katom-steps/s", self._n,
                         st["graph_ms"], st["model_ms"], st["read_ms"], st["katom_steps_per_s"])
        return self._result

    def stats(self) -> Dict[str, float]:
        """Mean milliseconds per evaluation of each part, and the atom-step rate."""
        n = max(self._n, 1)
        tot = self._t["total"]
        return {"evaluations": self._n, "graph_ms": 1e3 * self._t["graph"] / n, "model_ms": 1e3 * self._t["model"] / n,
                "read_ms": 1e3 * self._t["read"] / n, "katom_steps_per_s": (self.natoms * self._n / tot / 1e3)
                if tot > 0 else 0.0}

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
        elif c == ">TOTCHARGE":
            self.total_charge = float(comm.recv(1, "double")[0])
        elif c == "<COORDS":
            comm.send((self.coords / BOHR).reshape(-1).tolist(), "double")
        elif c == "<CELL":
            cell = np.zeros((3, 3)) if self.cell is None else self.cell
            comm.send((cell / BOHR).reshape(-1).tolist(), "double")
        elif c == "SCF":
            self._evaluate()
        elif c == "<ENERGY":
            comm.send([float(self._evaluate()["energy"].sum()) / HARTREE], "double")
        elif c == "<FORCES":
            comm.send((self._evaluate()["forces"] * (BOHR / HARTREE)).reshape(-1).tolist(), "double")
        elif c == "<STRESS":
            st = self._evaluate().get("stress") if self.cell is not None else None
            st = np.zeros(9) if st is None else -st.reshape(-1)      # pressure sign on the wire
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
