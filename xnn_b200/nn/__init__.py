"""Featurizers and small building blocks shared by the model families."""
from .cutoff import CosineCutoff, MollifierCutoff, PolynomialCutoff
from .radial import (BesselRBF, ExpNormalSmearing, GaussianRBF, SmoothBesselRBF,
                     make_radial_basis)

__all__ = ["BesselRBF", "CosineCutoff", "ExpNormalSmearing", "GaussianRBF", "MollifierCutoff",
           "PolynomialCutoff", "SmoothBesselRBF", "make_radial_basis"]
