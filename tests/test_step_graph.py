"""Skin-list MD steps (StepGraph) against direct evaluation on a fresh neighbour list, for a
fixed-topology force field and a message-passing model, and velocity-Verlet energy conservation."""
import pytest
import torch

from xnn_b200.data import collate, structure_to_graph
from xnn_b200.deploy.step_graph import StepGraph, VerletStepper
from xnn_b200.models.outputs import ForceStressOutput


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _butane_model(cutoff=4.0):
    from test_classical_ff import _butane
    from xnn_b200.ffnn.opls import OPLS
    from xnn_b200.ffnn.topology import MolecularTopology
    pos, z, types, bonds = _butane()
    return OPLS("oplsaa", MolecularTopology.from_bonds(types, bonds), cutoff=cutoff), torch.tensor(pos), torch.tensor(z)


def _direct(model, pos, z, cutoff, cell=None):
    s = {"pos": pos.detach().cpu(), "atomic_numbers": z.cpu()}
    if cell is not None:
        s["cell"], s["pbc"] = cell.cpu(), torch.tensor([True, True, True])
    return ForceStressOutput(model)(collate([structure_to_graph(s, cutoff)]).to(pos.device))


@pytest.mark.parametrize("periodic", [False, True])
def test_step_graph_matches_fresh_lists(periodic):
    model, pos, z = _butane_model()
    cell = torch.eye(3) * 9.0 if periodic else None
    sg = StepGraph(model, skin=1.0)
    g = torch.Generator().manual_seed(0)
    for k in range(6):
        p = pos + 0.12 * torch.randn(pos.shape, generator=g)
        s = {"pos": p, "atomic_numbers": z}
        if periodic:
            s["cell"], s["pbc"] = cell, torch.tensor([True, True, True])
        out, ref = sg(s), _direct(model, p, z, 4.0, cell)
        torch.testing.assert_close(out["energy"], ref["energy"].detach(), rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(out["forces"], ref["forces"].detach(), rtol=1e-10, atol=1e-10)
    assert sg.rebuilds < 6            # the skin list survived some steps


def test_step_graph_message_passing_model():
    from xnn_b200.models.schnet import SchNet
    torch.manual_seed(0)
    model = SchNet(n_features=8, n_interactions=2, n_rbf=6, cutoff=3.0)
    pos = torch.rand(10, 3) * 4.0
    z = torch.tensor([1, 6, 8, 1, 6, 8, 1, 6, 8, 1])
    sg = StepGraph(model, skin=0.8)
    for k in range(3):
        p = pos + 0.05 * k
        out, ref = sg({"pos": p, "atomic_numbers": z}), _direct(model, p, z, 3.0)
        torch.testing.assert_close(out["energy"], ref["energy"].detach(), rtol=1e-9, atol=1e-9)
        torch.testing.assert_close(out["forces"], ref["forces"].detach(), rtol=1e-9, atol=1e-9)


def test_verlet_conserves_energy():
    model, pos, z = _butane_model(cutoff=6.0)
    sg = StepGraph(model, skin=1.0)
    torch.manual_seed(1)
    md = VerletStepper(sg, {"pos": pos, "atomic_numbers": z}, model.masses, dt=0.25,
                       velocities=0.005 * torch.randn(pos.shape))
    e0 = float(md.out["energy"]) + float(md.kinetic_energy())
    md.run(40)
    e1 = float(md.out["energy"]) + float(md.kinetic_energy())
    assert abs(e1 - e0) < 2e-3 * max(1.0, abs(e0))


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["opls", "schnet"])
def test_step_graph_replay_on_gpu(kind):
    dev = torch.device("cuda")
    if kind == "opls":
        model, pos, z = _butane_model()
        cutoff = 4.0
    else:
        from xnn_b200.models.schnet import SchNet
        torch.manual_seed(0)
        model, cutoff = SchNet(n_features=8, n_interactions=2, n_rbf=6, cutoff=3.0), 3.0
        pos, z = torch.rand(12, 3) * 4.0, torch.tensor([1, 6, 8] * 4)
    model = model.to(dev)
    sg = StepGraph(model, skin=1.0, warmup=1)
    g = torch.Generator().manual_seed(0)
    for k in range(5):
        p = (pos + 0.1 * torch.randn(pos.shape, generator=g)).to(dev)
        out, ref = sg({"pos": p, "atomic_numbers": z.to(dev)}), _direct(model, p, z.to(dev), cutoff)
        torch.testing.assert_close(out["energy"], ref["energy"].detach(), rtol=1e-9, atol=1e-9)
        torch.testing.assert_close(out["forces"], ref["forces"].detach(), rtol=1e-9, atol=1e-9)
    assert sg.captures >= 1 and sg._graphed is not None
    sg.release()
