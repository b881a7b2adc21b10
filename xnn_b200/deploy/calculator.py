"""ASE calculator over any potential of this package.

Behaviour follows the reference's ``XNNCalculator`` (``src/xnn/common/deploy/ase_calculator.py:26``):
an ``Atoms``-like object becomes an :class:`~xnn_b200.data.AtomicGraph` with float64 positions
and cell whatever the model's dtype (the model computes in its own dtype through
``compute_dtype``), the neighbour list uses the model's cutoff, and ``results`` holds the energy
(eV), forces (eV/A), the Voigt stress ``[xx, yy, zz, yz, xz, xy]`` of periodic structures and
LES / model charges and dipoles when the model predicts them. ``cuda_graph=True`` replays the
evaluation as one CUDA graph (:class:`~xnn_b200.deploy.graphed_eval.GraphedEvaluation`).

ASE is optional: when it is installed the class is an ``ase.calculators.calculator.Calculator``;
without it a minimal base with the same ``get_*`` methods accepts any object exposing
``get_positions``, ``get_atomic_numbers``, ``get_cell``, ``pbc`` and ``info``.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from ..data.dataset import structure_to_graph

try:  # pragma: no cover - depends on the environment
    from ase.calculators.calculator import Calculator, all_changes
    HAS_ASE = True
except ImportError:
    HAS_ASE = False
    all_changes = ["positions", "numbers", "cell", "pbc", "initial_charges", "initial_magmoms"]

    class Calculator:  # minimal stand-in with the ASE calculator protocol used here
        implemented_properties = []

        def __init__(self, **kwargs):
            self.results = {}
            self.atoms = None
            self.parameters = dict(kwargs)

        def calculate(self, atoms=None, properties=("energy",), system_changes=all_changes):
            if atoms is not None:
                self.atoms = atoms
            self.results = {}

        def get_property(self, name, atoms=None, allow_calculation=True):
            atoms = atoms if atoms is not None else self.atoms
            self.calculate(atoms, [name], all_changes)
            return self.results[name]

        def get_potential_energy(self, atoms=None, force_consistent=False):
            return self.get_property("energy", atoms)

        def get_forces(self, atoms=None):
            return self.get_property("forces", atoms)

        def get_stress(self, atoms=None):
            return self.get_property("stress", atoms)


def _float_dtype(model) -> torch.dtype:
    for p in list(model.parameters()) + list(model.buffers()):
        if p.is_floating_point():
            return p.dtype
    return torch.get_default_dtype()


class XNNCalculator(Calculator):
    implemented_properties = ["energy", "forces", "stress", "charges", "dipole"]

    def __init__(self, model, cutoff: Optional[float] = None, device: str = "cpu", cuda_graph: bool = False,
                 **kwargs):
        super().__init__(**kwargs)
        from ..models.outputs import ForceStressOutput
        if not hasattr(model, "compute_forces"):
            model = ForceStressOutput(model, compute_stress=True)
        self.model = model.to(device).eval()
        self.dtype = _float_dtype(self.model)
        self.cutoff = float(cutoff if cutoff is not None else self.model.cutoff)
        self.device = device
        self._graphed = None
        if cuda_graph and torch.device(device).type == "cuda":
            from .graphed_eval import GraphedEvaluation
            self._graphed = GraphedEvaluation(self.model)

    @classmethod
    def from_pretrained(cls, source, device: str = "cpu", **kwargs) -> "XNNCalculator":
        from ..hub import from_pretrained
        model = from_pretrained(source)
        return cls(model, cutoff=model.cutoff, device=device, **kwargs)

    def calculate(self, atoms=None, properties=("energy",), system_changes=all_changes):
        super().calculate(atoms, properties, system_changes)
        atoms = atoms if atoms is not None else self.atoms
        pbc = np.asarray(atoms.pbc if not callable(getattr(atoms, "pbc", None)) else atoms.get_pbc(), dtype=bool)
        struct = {"pos": torch.as_tensor(np.asarray(atoms.get_positions()), dtype=torch.float64),
                  "atomic_numbers": np.asarray(atoms.get_atomic_numbers()),
                  "cell": torch.as_tensor(np.asarray(atoms.get_cell()), dtype=torch.float64) if pbc.any() else None,
                  "pbc": pbc}
        info = getattr(atoms, "info", {}) or {}
        for key in ("total_charge", "charge"):
            if key in info:
                struct["total_charge"] = float(info[key])
                break
        for key in ("spin_multiplicity", "multiplicity"):
            if key in info:
                struct["spin_multiplicity"] = float(info[key])
                break
        g = structure_to_graph(struct, self.cutoff, device=self.device)
        if self.dtype != g.pos.dtype:
            g.compute_dtype = self.dtype
        out = self._graphed(g) if self._graphed is not None else self.model(g)
        self.results["energy"] = float(out["energy"].sum().detach())
        if "forces" in out:
            self.results["forces"] = out["forces"].detach().cpu().numpy()
        if "stress" in out and pbc.any():
            s = out["stress"][0].detach().cpu().numpy()
            self.results["stress"] = np.array([s[0, 0], s[1, 1], s[2, 2], s[1, 2], s[0, 2], s[0, 1]])
        if "charges" in out:
            self.results["charges"] = out["charges"].detach().cpu().numpy()
        elif "les_charges" in out:
            self.results["charges"] = out["les_charges"].detach().cpu().numpy()
        if "dipole" in out:
            self.results["dipole"] = out["dipole"][0].detach().cpu().numpy()
        elif "les_dipole" in out and not pbc.any():
            self.results["dipole"] = out["les_dipole"][0].detach().cpu().numpy()
