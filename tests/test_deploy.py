"""Deployment: ASE-protocol calculator, LAMMPS/TorchScript archive, MDI engine handlers."""
import numpy as np
import pytest
import torch

from xnn_b200.data import structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.mace import MACE


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _model():
    torch.manual_seed(0)
    return MACE(species=[1, 6, 7, 8, 9, 16, 17], cutoff=4.5, num_channels=8, n_rbf=6, num_interactions=2,
                max_ell=2, correlation=2, avg_num_neighbors=6.0)


class _Atoms:
    """The part of ase.Atoms the calculator reads."""

    def __init__(self, s):
        self._pos = s["pos"].numpy()
        self._z = s["atomic_numbers"].numpy()
        self._cell = s["cell"].numpy() if s.get("cell") is not None else np.zeros((3, 3))
        self.pbc = np.asarray(s.get("pbc", [False] * 3), dtype=bool) if s.get("cell") is not None else np.zeros(3, bool)
        self.info = {}

    def get_positions(self):
        return self._pos

    def get_atomic_numbers(self):
        return self._z

    def get_cell(self):
        return self._cell


def test_calculator_matches_model():
    from xnn_b200.deploy.calculator import XNNCalculator
    m = _model()
    calc = XNNCalculator(m)
    for s in (synthetic.organic_molecules(1, seed=2, labels=False)[0],
              synthetic.triclinic_crystals(1, seed=1, labels=False)[0]):
        if s.get("cell") is not None:
            s["atomic_numbers"] = torch.full_like(s["atomic_numbers"], 6)
        atoms = _Atoms(s)
        e = calc.get_potential_energy(atoms)
        f = calc.get_forces(atoms)
        ref = ForceStressOutput(m, compute_stress=True)(structure_to_graph(s, 4.5))
        assert abs(e - float(ref["energy"].sum())) < 1e-10
        np.testing.assert_allclose(f, ref["forces"].detach().numpy(), rtol=1e-9, atol=1e-10)
        if s.get("cell") is not None:
            st = calc.get_stress(atoms)
            r = ref["stress"][0].detach().numpy()
            np.testing.assert_allclose(st, [r[0, 0], r[1, 1], r[2, 2], r[1, 2], r[0, 2], r[0, 1]], atol=1e-10)


def test_lammps_archive_round_trip(tmp_path):
    from xnn_b200.deploy.lammps import export_to_lammps, load_lammps
    m = _model()
    path = export_to_lammps(m, 4.5, str(tmp_path / "model.pt"), metadata={"note": "test"})
    mod, extra = load_lammps(path)
    assert float(extra["cutoff"]) == 4.5
    for s in (synthetic.organic_molecules(1, seed=7, labels=False)[0],
              synthetic.triclinic_crystals(1, seed=3, labels=False)[0]):
        if s.get("cell") is not None:
            s["atomic_numbers"] = torch.full_like(s["atomic_numbers"], 8)
        g = structure_to_graph(s, 4.5)
        cell = g.cell[0] if g.cell is not None else torch.zeros(3, 3)
        out = mod(g.pos, g.edge_index, g.cell_shifts, g.atomic_numbers, cell)
        m.set_use_fast(False)
        ref = ForceStressOutput(m)(g.clone())
        torch.testing.assert_close(out["total_energy"], ref["energy"].reshape(1), rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(out["forces"], ref["forces"], rtol=1e-9, atol=1e-10)


def test_torchscript_standalone_and_openmm(tmp_path):
    from xnn_b200.deploy.torchscript import export_torchscript, openmm_force
    m = _model()
    path = export_torchscript(m, str(tmp_path / "ts.pt"))
    mod = torch.jit.load(path)
    m.set_use_fast(False)
    s = synthetic.triclinic_crystals(1, seed=4, labels=False)[0]
    s["atomic_numbers"] = torch.full_like(s["atomic_numbers"], 6)
    g = structure_to_graph(s, 4.5)
    out = mod(g.pos, g.atomic_numbers, g.cell[0], g.pbc[0])
    ref = ForceStressOutput(m, compute_stress=True)(g.clone())
    torch.testing.assert_close(out["energy"], ref["energy"].reshape(1), rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(out["forces"], ref["forces"], rtol=1e-9, atol=1e-10)
    torch.testing.assert_close(out["stress"], ref["stress"], rtol=1e-9, atol=1e-10)
    mol = synthetic.organic_molecules(1, seed=9, labels=False)[0]
    gm = structure_to_graph(mol, 4.5)
    f = openmm_force(m, gm.atomic_numbers)
    e_kj = f(gm.pos / 10.0)
    e_ref = ForceStressOutput(m)(gm.clone())["energy"]
    torch.testing.assert_close(e_kj / 96.48533212331002, e_ref.reshape(()), rtol=1e-10, atol=1e-10)


def test_mdi_engine_protocol():
    from xnn_b200.deploy.mdi_engine import MDIEngine
    from xnn_b200.models.dispersion import BOHR, HARTREE
    m = _model()
    s = synthetic.organic_molecules(1, seed=12, labels=False)[0]
    n = s["pos"].shape[0]

    class Comm:
        def __init__(self, script):
            self.script = list(script)
            self.sent = []

        def recv_command(self):
            return self.script.pop(0)

        def recv(self, count, kind):
            v = self.script.pop(0)
            assert len(v) == count
            return v

        def send(self, values, kind):
            self.sent.append(list(values))

    comm = Comm([">NATOMS", [n], ">ELEMENTS", s["atomic_numbers"].tolist(),
                 ">COORDS", (s["pos"] / BOHR).reshape(-1).tolist(), "<ENERGY", "<FORCES", "EXIT"])
    MDIEngine(m).serve(comm)
    ref = ForceStressOutput(m)(structure_to_graph(s, 4.5))
    assert abs(comm.sent[0][0] * HARTREE - float(ref["energy"].sum().detach())) < 1e-9
    np.testing.assert_allclose(np.array(comm.sent[1]).reshape(-1, 3) * HARTREE / BOHR,
                               ref["forces"].detach().numpy(), rtol=1e-8, atol=1e-9)


def test_mdi_engine_cell_charge_stress_and_stats():
    from xnn_b200.deploy.mdi_engine import MDIEngine
    from xnn_b200.models.dispersion import BOHR, HARTREE
    m = _model()
    s = synthetic.triclinic_crystals(1, seed=3, n_min=10, n_max=14, z_max=17, labels=False)[0]
    n = s["pos"].shape[0]

    class Comm:
        def __init__(self, script):
            self.script, self.sent = list(script), []

        def recv_command(self):
            return self.script.pop(0)

        def recv(self, count, kind):
            return self.script.pop(0)

        def send(self, values, kind):
            self.sent.append(list(values))

    comm = Comm([">NATOMS", [n], ">ELEMENTS", s["atomic_numbers"].tolist(), ">TOTCHARGE", [0.0],
                 ">CELL", (s["cell"] / BOHR).reshape(-1).tolist(), ">COORDS", (s["pos"] / BOHR).reshape(-1).tolist(),
                 "SCF", "<ENERGY", "<STRESS", "<CELL", "EXIT"])
    eng = MDIEngine(m)
    eng.serve(comm)
    ref = ForceStressOutput(m, compute_stress=True)(structure_to_graph(s, 4.5))
    assert abs(comm.sent[0][0] * HARTREE - float(ref["energy"].sum().detach())) < 1e-9
    np.testing.assert_allclose(-np.array(comm.sent[1]).reshape(3, 3) * HARTREE / BOHR ** 3,
                               ref["stress"][0].detach().numpy(), rtol=1e-7, atol=1e-10)
    np.testing.assert_allclose(np.array(comm.sent[2]).reshape(3, 3) * BOHR, s["cell"].numpy(), rtol=1e-12)
    assert eng.stats()["evaluations"] == 1


def test_openmm_ml_potential_on_a_subset(monkeypatch):
    """MLPotential("xnn_b200") through the factory, with stand-ins for OpenMM's topology and system and
    for openmm-torch's TorchForce: the force acts on the chosen atoms only."""
    import sys
    import types

    from xnn_b200.deploy.openmm_ml import XNNPotentialImplFactory

    class _TorchForce:
        def __init__(self, module):
            self.module, self.group, self.periodic = module, None, None

        def setForceGroup(self, g):
            self.group = g

        def setUsesPeriodicBoundaryConditions(self, p):
            self.periodic = p

    monkeypatch.setitem(sys.modules, "openmmtorch", types.SimpleNamespace(TorchForce=_TorchForce))
    mol = synthetic.organic_molecules(1, seed=9, labels=False)[0]
    z = mol["atomic_numbers"].tolist()
    water = [8, 1, 1]
    Atom = types.SimpleNamespace
    atoms = [Atom(element=Atom(atomic_number=int(a))) for a in water + z]
    topology = types.SimpleNamespace(atoms=lambda: iter(atoms), getPeriodicBoxVectors=lambda: None)
    system = types.SimpleNamespace(forces=[])
    system.addForce = system.forces.append
    m = _model()
    with pytest.raises(ValueError):
        XNNPotentialImplFactory().createImpl("xnn_b200")
    impl = XNNPotentialImplFactory().createImpl("xnn_b200", model=m)
    sub = list(range(3, 3 + len(z)))
    impl.addForces(topology, system, sub, 2)
    (force,) = system.forces
    assert force.group == 2 and force.periodic is False
    pos = torch.cat([torch.zeros(3, 3), mol["pos"]], 0) / 10.0
    e_kj = force.module(pos)
    m.set_use_fast(False)
    e_ref = ForceStressOutput(m)(structure_to_graph(mol, 4.5))["energy"]
    torch.testing.assert_close(e_kj / 96.48533212331002, e_ref.reshape(()), rtol=1e-10, atol=1e-10)
