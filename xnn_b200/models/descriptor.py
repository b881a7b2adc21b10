"""Descriptor potentials: an invariant per-atom featurizer feeding one network per element
(HDNNP / ANI), plus per-element self energies.

Parameter names and the element-network layout (``element_nets.nets[str(Z)]`` as ``nn.Sequential``
of linear layers and activations, ``_self_energies_by_z``) follow the reference
(``src/xnn/dnn/models/base.py:76-498``) so that weights transplant. The atoms are sorted by element
once (one host read of the block sizes) and every network runs on its contiguous block.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple, Union

import torch
from torch import Tensor, nn

from ..data import AtomicGraph
from ..nn.blocks import make_activation
from .base import InteratomicPotential


class ElementNetworks(nn.Module):
    def __init__(self, species: Sequence[int], input_dim: Union[int, dict], hidden=(64, 64), activation="silu",
                 bias: bool = True, extra_inputs: int = 0, n_outputs: int = 1):
        super().__init__()
        self.species = [int(z) for z in species]
        self.n_outputs = int(n_outputs)
        self.input_dims = {z: int(input_dim[z]) if isinstance(input_dim, dict) else int(input_dim)
                           for z in self.species}
        self.extra_inputs = int(extra_inputs)
        code = torch.full((max(self.species) + 1,), len(self.species), dtype=torch.long)
        for k, z in enumerate(self.species):
            code[z] = k
        self.register_buffer("_code_of_z", code, persistent=False)
        self.nets = nn.ModuleDict()
        for z in self.species:
            widths = list(hidden[z] if isinstance(hidden, dict) else hidden)
            acts = activation[z] if isinstance(activation, dict) else activation
            if isinstance(acts, (str, nn.Module)):
                acts = [acts] * len(widths) + [None]
            acts = list(acts)
            if len(acts) != len(widths) + 1:
                raise ValueError(f"element {z}: {len(acts)} activations for {len(widths)} hidden layers and the "
                                 f"output layer (need {len(widths) + 1})")
            layers, d = [], self.input_dims[z] + self.extra_inputs
            for h, act in zip(widths + [self.n_outputs], acts):
                layers.append(nn.Linear(d, h, bias=bias))
                if act is not None and not (isinstance(act, str) and act.lower() == "linear" and h == self.n_outputs):
                    layers.append(make_activation(act))
                d = h
            self.nets[str(z)] = nn.Sequential(*layers)

    def element_code(self, z: Tensor) -> Tensor:
        m = self._code_of_z.shape[0]
        code = self._code_of_z[z.clamp(max=m - 1)]
        return torch.where(z < m, code, torch.full_like(code, len(self.species)))

    def plan(self, z: Tensor) -> Tuple[Tensor, List[int]]:
        code = self.element_code(z)
        order = torch.argsort(code, stable=True)
        return order, torch.bincount(code, minlength=len(self.species) + 1).tolist()

    def forward(self, desc: Tensor, atomic_numbers: Tensor, extra: Optional[Tensor] = None, plan=None) -> Tensor:
        order, sizes = self.plan(atomic_numbers) if plan is None else plan
        n = desc.shape[0]
        x_all = desc.index_select(0, order)
        e_all = (extra.reshape(n, -1).index_select(0, order)
                 if self.extra_inputs > 0 and extra is not None else None)
        blocks = x_all.split(sizes)
        e_blocks = e_all.split(sizes) if e_all is not None else None
        pieces = []
        for k, z in enumerate(self.species):
            if sizes[k] == 0:
                continue
            x = blocks[k]
            width = self.input_dims[z]
            if width < x.shape[1]:
                x = x[:, :width]
            if e_blocks is not None:
                x = torch.cat([x, e_blocks[k].to(x.dtype)], -1)
            y = self.nets[str(z)](x)
            pieces.append(y.squeeze(-1) if self.n_outputs == 1 else y)
        rest = sizes[len(self.species)]
        shape = (rest,) if self.n_outputs == 1 else (rest, self.n_outputs)
        if rest:
            pieces.append(desc.new_zeros(shape))
        values = torch.cat(pieces) if pieces else desc.new_zeros(shape)
        out = desc.new_zeros((n,) if self.n_outputs == 1 else (n, self.n_outputs))
        return out.index_copy(0, order, values)


class DescriptorPotential(InteratomicPotential):
    head_modules = ("element_nets", "_self_energies_by_z")

    def __init__(self, featurizer: nn.Module, species: Sequence[int], hidden=(64, 64), activation="silu",
                 bias: bool = True, atomic_energies: Optional[Sequence[float]] = None, extra_inputs: int = 0):
        super().__init__()
        self.featurizer = featurizer
        self.cutoff = float(featurizer.cutoff)
        self.node_feature_dim = featurizer.output_dim
        self.species = [int(z) for z in species]
        dims = getattr(featurizer, "n_features", None) or featurizer.output_dim
        self.element_nets = ElementNetworks(species, dims, hidden, activation, bias, extra_inputs)
        sae = torch.zeros(max(self.species) + 1)
        if atomic_energies is not None:
            ae = torch.as_tensor(atomic_energies, dtype=sae.dtype)
            if ae.numel() != len(self.species):
                raise ValueError(f"atomic_energies: got {ae.numel()} values for {len(self.species)} species")
            for z, e in zip(self.species, ae.tolist()):
                sae[z] = e
        self.register_buffer("_self_energies_by_z", sae)

    def node_features_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor):
        desc = self.featurizer.compute(atomic_numbers, edge_index, edge_vec, atomic_numbers.shape[0])
        return desc, self.element_nets(desc, atomic_numbers) + self._self_energies_by_z[atomic_numbers]

    def node_energy(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor) -> Tensor:
        return self.node_features_energy(atomic_numbers, edge_index, edge_vec)[1]

    def forward(self, data: AtomicGraph) -> dict:
        desc = self.featurizer(data)
        ne = self.element_nets(desc, data.atomic_numbers) + self._self_energies_by_z[data.atomic_numbers]
        return {"node_energy": ne, "energy": self.aggregate_energy(ne, data), "node_features": desc}
