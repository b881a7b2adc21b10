"""The ``"xnn_b200"`` potential of openmm-ml: ``MLPotential("xnn_b200", model=...)``.

openmm-ml finds potentials through the ``openmmml.potentials`` entry point; this module provides the
factory it calls (``createImpl``) and the implementation whose ``addForces`` puts the model into an
OpenMM ``System`` as an openmm-torch ``TorchForce``, on all atoms or on a subset (ML/MM, the rest of
the system keeping its classical forces). The model is an ``nn.Module``, a model directory or a hub
name (:func:`xnn_b200.hub.from_pretrained`); positions in nm and energies in kJ/mol are converted by
:class:`~xnn_b200.deploy.torchscript.OpenMMForce`. openmm and openmm-torch are imported on use.

Parity: the reference's ``XNNPotentialImplFactory`` (``src/xnn/common/deploy/openmm_force.py:241``) and
its entry point (``pyproject.toml:146``).
"""
from __future__ import annotations

from typing import Iterable, Optional

from torch import nn


def _resolve(model) -> nn.Module:
    if isinstance(model, nn.Module):
        return model
    from ..hub import from_pretrained
    return from_pretrained(model)


class XNNPotentialImpl:
    """``addForces(topology, system, atoms, forceGroup)`` as openmm-ml calls it."""

    def __init__(self, model, **options):
        self.model = _resolve(model)
        self.options = dict(options)

    def addForces(self, topology, system, atoms: Optional[Iterable[int]], forceGroup: int, **args) -> None:
        import openmmtorch

        from .torchscript import openmm_force
        all_atoms = list(topology.atoms())
        idx = list(range(len(all_atoms))) if atoms is None else [int(a) for a in atoms]
        z = [all_atoms[i].element.atomic_number for i in idx]
        periodic = topology.getPeriodicBoxVectors() is not None
        module = openmm_force(self.model, z, periodic=periodic, atoms=None if atoms is None else idx)
        force = openmmtorch.TorchForce(module)
        force.setForceGroup(int(forceGroup))
        if hasattr(force, "setUsesPeriodicBoundaryConditions"):
            force.setUsesPeriodicBoundaryConditions(periodic)
        system.addForce(force)


class XNNPotentialImplFactory:
    """The factory openmm-ml calls for ``MLPotential("xnn_b200", model=...)``."""

    def createImpl(self, name: str, model=None, **args) -> XNNPotentialImpl:
        if model is None:
            raise ValueError('MLPotential("xnn_b200") needs model=: a model, a model directory or a hub name')
        return XNNPotentialImpl(model, **args)


__all__ = ["XNNPotentialImpl", "XNNPotentialImplFactory"]
