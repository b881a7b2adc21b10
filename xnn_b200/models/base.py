"""The model contract and the species bookkeeping shared by the graph potentials.

Every model maps an :class:`~xnn_b200.data.AtomicGraph` to at least
``{"node_energy": (N,), "energy": (B,)}`` (``src/xnn/common/models/base.py:24-180``);
forces and stress are added uniformly by
:class:`~xnn_b200.models.outputs.ForceStressOutput`. ``receptive_field`` sizes the
ghost shell of a domain-decomposed evaluation; ``refreshes_ghosts`` says the model
refreshes ghost features between layers; ``head_modules`` names one readout head.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from ..data import AtomicGraph
from ..ops.scatter import structure_sum


class InteratomicPotential(nn.Module):
    head_modules: tuple = ()
    refreshes_ghosts: bool = False

    def forward(self, data: AtomicGraph) -> dict:  # pragma: no cover - abstract
        raise NotImplementedError

    @classmethod
    def from_config(cls, cfg) -> "InteratomicPotential":  # pragma: no cover - abstract
        raise NotImplementedError

    @classmethod
    def from_pretrained(cls, source, **kwargs) -> "InteratomicPotential":
        from ..hub import from_pretrained
        model = from_pretrained(source, wrap=False, **kwargs)
        core = getattr(model, "model", model)
        if not isinstance(model, cls) and not isinstance(core, cls):
            raise TypeError(f"{source!r} holds a {type(core).__name__}, not a {cls.__name__}")
        return model

    def receptive_field(self) -> Optional[float]:
        return None

    def aggregate_energy(self, node_energy: Tensor, data: AtomicGraph) -> Tensor:
        """Float64 per-structure sums of the per-atom energies."""
        return structure_sum(node_energy, data.batch, data.num_graphs)


class GNNPotential(InteratomicPotential):
    """Species table (``z_to_index``), one-hot node attributes and ``atom_ref`` energies."""

    def __init__(self, species, cutoff: float):
        super().__init__()
        self.species = [int(z) for z in species]
        self.cutoff = float(cutoff)
        z_to_index = torch.full((200,), -1, dtype=torch.long)
        for i, z in enumerate(self.species):
            z_to_index[z] = i
        self.register_buffer("z_to_index", z_to_index)
        self.atom_ref = nn.Embedding(200, 1)
        nn.init.zeros_(self.atom_ref.weight)

    def set_atomic_energies(self, values) -> None:
        ae = torch.as_tensor(values, dtype=self.atom_ref.weight.dtype)
        if ae.numel() != len(self.species):
            raise ValueError(f"got {ae.numel()} atomic energies for {len(self.species)} species")
        with torch.no_grad():
            self.atom_ref.weight[torch.tensor(self.species), 0] = ae

    def element_index(self, atomic_numbers: Tensor) -> Tensor:
        return self.z_to_index[atomic_numbers]

    def node_attr(self, atomic_numbers: Tensor) -> Tensor:
        idx = self.z_to_index[atomic_numbers]
        return F.one_hot(idx.clamp(min=0), len(self.species)).to(self.atom_ref.weight.dtype)
