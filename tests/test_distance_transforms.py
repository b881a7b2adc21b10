"""Agnesi and Soft distance warps: closed forms at hand-computed points, limits, and MACE with
the warp on (energy and forces by autograd)."""
import math

import torch

from xnn_b200.nn.transforms import DISTANCE_TRANSFORMS, AgnesiDistanceTransform, SoftDistanceTransform


def _edge(z1, z2, r):
    z = torch.tensor([z1, z2])
    ei = torch.tensor([[0], [1]])
    return torch.tensor([r], dtype=torch.float64), z, ei


def test_agnesi_closed_form():
    r, z, ei = _edge(6, 8, 1.3)                      # C 0.76, O 0.66 -> r0 = 0.71
    u = 1.3 / 0.71
    a, q, p = 1.0805, 0.9183, 4.5791
    want = 1.0 / (1.0 + a * u ** q / (1.0 + u ** (q - p)))
    got = AgnesiDistanceTransform()(r, z, ei)
    assert abs(float(got) - want) < 1e-12
    # decreasing in r, 1 at r -> 0
    rr = torch.linspace(0.05, 6.0, 200, dtype=torch.float64)
    t = AgnesiDistanceTransform()(rr, z, ei.expand(2, 200))
    assert bool((t[1:] < t[:-1]).all()) and float(t[0]) > 0.9


def test_soft_clamp_limits():
    T = SoftDistanceTransform()
    s = 0.31 + 0.76                                   # H-C sum of radii
    r, z, ei = _edge(1, 6, 0.2)
    assert abs(float(T(r, z, ei)) - 0.75 * s) < 1e-3  # floor far below the switch
    r, z, ei = _edge(1, 6, 4.0)
    assert abs(float(T(r, z, ei)) - 4.0) < 1e-9      # identity far above
    mid = 0.5 * (0.75 * s + 4.0 / 3.0 * s)
    r, z, ei = _edge(1, 6, mid)
    assert abs(float(T(r, z, ei)) - (0.75 * s + 0.5 * (mid - 0.75 * s))) < 1e-12
    assert math.isclose(float(T.alpha), 4.0)


def test_registry_and_mace_with_agnesi():
    assert set(DISTANCE_TRANSFORMS) == {None, "None", "Agnesi", "Soft"}
    from xnn_b200.data import collate, structure_to_graph, synthetic
    from xnn_b200.models import ForceStressOutput
    from xnn_b200.models.mace import MACE
    torch.manual_seed(0)
    model = MACE(species=[1, 6, 7, 8], cutoff=4.0, num_channels=8, max_ell=2, correlation=2,
                 distance_transform="Agnesi").double()
    assert "distance_transform.covalent_radii" in model.state_dict()
    mols = synthetic.organic_molecules(2, seed=1, n_min=6, n_max=10)
    b = collate([structure_to_graph(s, 4.0) for s in mols])
    out = ForceStressOutput(model)(b)
    assert torch.isfinite(out["energy"]).all() and torch.isfinite(out["forces"]).all()
