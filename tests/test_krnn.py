"""sGDML pieces on their own: the Matern kernel derivatives and the symmetry search."""
import numpy as np
import torch

from xnn_b200.krnn.kernels import Matern
from xnn_b200.krnn.permutations import find_permutations


def test_matern_derivative_forms():
    k = Matern(2.5, 3)
    r = torch.linspace(0.1, 4.0, 50, dtype=torch.float64, requires_grad=True)
    (dk,) = torch.autograd.grad(k.k(r).sum(), r, create_graph=True)
    torch.testing.assert_close(k.g(r), -dk / r)
    (dg,) = torch.autograd.grad(k.g(r).sum(), r)
    torch.testing.assert_close(k.t_of(r).detach(), dg / r.detach())


def test_symmetry_search_finds_the_hydrogen_swap():
    rng = np.random.default_rng(0)
    base = np.array([[0.0, 0.0, 0.0], [0.96, 0.0, 0.0], [-0.24, 0.93, 0.0]])
    geoms = []
    for k in range(6):
        g = base + 0.02 * rng.standard_normal((3, 3))
        geoms.append(g[[0, 2, 1]] if k % 2 else g)      # half of them with the hydrogens swapped
    perms = find_permutations(np.stack(geoms), np.array([8, 1, 1]))
    assert {tuple(p) for p in perms.tolist()} == {(0, 1, 2), (0, 2, 1)}
