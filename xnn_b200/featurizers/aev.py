"""The ANI atomic environment vector: radial and angular symmetry functions concatenated
(Smith et al., Chem. Sci. 8, 3192, 2017), with the ANI-1, ANI-1x and ANI-2x grids of the
reference (``src/xnn/dnn/featurizers/aev.py:53-239``) as class methods."""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
from torch import Tensor, nn

from .symmetry_functions import AngularSymmetryFunctions, RadialSymmetryFunctions

ANI_SPECIES = [1, 6, 7, 8]
ANI2X_SPECIES = [1, 6, 7, 8, 16, 9, 17]


def even_shifts(cutoff: float, n: int, start: float = 0.9) -> tuple:
    step = (cutoff - start) / n
    return tuple(start + step * i for i in range(n))


def angle_shifts(n: int) -> tuple:
    return tuple(math.pi / (2 * n) * (2 * i + 1) for i in range(n))


class AEV(nn.Module):
    def __init__(self, species, radial_cutoff: float = 5.2, angular_cutoff: float = 3.5, radial_etas=(16.0,),
                 radial_rs=even_shifts(5.2, 16), angular_etas=(8.0,), angular_zetas=(32.0,),
                 angular_rs=even_shifts(3.5, 4), angular_theta_s=angle_shifts(8), radial_prefactor: float = 0.25,
                 angular_cos_factor: float = 0.95):
        super().__init__()
        self.species = [int(z) for z in species]
        self.radial = RadialSymmetryFunctions(species, radial_cutoff, etas=radial_etas, rs=radial_rs,
                                              prefactor=radial_prefactor)
        self.angular = AngularSymmetryFunctions(species, angular_cutoff, etas=angular_etas, zetas=angular_zetas,
                                                rs=angular_rs, theta_s=angular_theta_s, cos_factor=angular_cos_factor)
        self.cutoff = max(float(radial_cutoff), float(angular_cutoff))

    @classmethod
    def ani1x(cls, species=ANI_SPECIES) -> "AEV":
        return cls(species, 5.2, 3.5, (16.0,), even_shifts(5.2, 16), (8.0,), (32.0,), even_shifts(3.5, 4),
                   angle_shifts(8))

    @classmethod
    def ani2x(cls, species=ANI2X_SPECIES) -> "AEV":
        return cls(species, 5.1, 3.5, (19.7,), even_shifts(5.1, 16, start=0.8), (12.5,), (14.1,),
                   even_shifts(3.5, 8, start=0.8), angle_shifts(4))

    @classmethod
    def ani1(cls, species=ANI_SPECIES) -> "AEV":
        return cls(species, 4.6, 3.1, (16.0,), even_shifts(4.6, 32), (8.0,), (8.0,), even_shifts(3.1, 8),
                   angle_shifts(8))

    @property
    def output_dim(self) -> int:
        return self.radial.output_dim + self.angular.output_dim

    def forward(self, data) -> Tensor:
        return self.compute(data.atomic_numbers, data.edge_index, data.edge_vectors(), data.num_nodes)

    def compute(self, atomic_numbers: Tensor, edge_index: Tensor, edge_vec: Tensor, num_nodes: int,
                triplets: Optional[Tuple[Tensor, Tensor]] = None) -> Tensor:
        r = torch.linalg.norm(edge_vec, dim=-1)
        return torch.cat([self.radial.compute(atomic_numbers, edge_index, edge_vec, num_nodes, r),
                          self.angular.compute(atomic_numbers, edge_index, edge_vec, num_nodes, r, triplets)], -1)
