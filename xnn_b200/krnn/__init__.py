"""Kernel-ridge force fields: the Matern kernel, inverse-distance descriptors, the sGDML fit,
symmetry (permutation) search and the sGDML model-file reader."""
