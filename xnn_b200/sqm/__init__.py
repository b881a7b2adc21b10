"""Semi-empirical quantum chemistry: NDDO Hamiltonians (PM3) on batched dense SCF."""
from .nddo import NDDO, PM3, amide_torsions
from .parameters import NDDOParameters, load_parameters, save_parameters

__all__ = ["NDDO", "PM3", "NDDOParameters", "amide_torsions", "load_parameters", "save_parameters"]
