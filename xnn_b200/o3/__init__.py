"""Equivariant primitives of O(3): irreps, spherical harmonics, coupling tensors, linear maps
and tensor products, with e3nn's conventions and parameter layouts (the reference builds its
equivariant models on e3nn, ``src/xnn/gnn/models/blocks.py``)."""
from ._fcnet import FullyConnectedNet, normalize2mom
from ._irreps import Irrep, Irreps, MulIr
from ._linear import Linear
from ._s2grid import FromS2Grid, ToS2Grid
from ._sh import SphericalHarmonics, spherical_harmonics
from ._tp import FullyConnectedTensorProduct, Instruction, TensorProduct
from ._wigner import su2_clebsch_gordan, wigner_3j

__all__ = ["FullyConnectedNet", "FullyConnectedTensorProduct", "Instruction", "Irrep", "Irreps",
           "FromS2Grid", "Linear", "MulIr", "SphericalHarmonics", "TensorProduct", "ToS2Grid", "normalize2mom",
           "spherical_harmonics", "su2_clebsch_gordan", "wigner_3j"]
