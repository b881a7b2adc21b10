"""Standalone invariant featurizers: atom-centred symmetry functions, the ANI AEV and the
Behler-Parrinello ACSF."""
from .symmetry_functions import AngularSymmetryFunctions, RadialSymmetryFunctions  # noqa: F401
from .aev import AEV, ANI_SPECIES, ANI2X_SPECIES  # noqa: F401
