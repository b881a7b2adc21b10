"""Classical fixed-topology force fields against the reference framework: the ``.frc`` reader, the
derived topology and the energies, forces and stress of the same library on the same conformers."""
import math

import pytest
import torch

from ref_oracle import ref_module
from xnn_b200.data import collate, structure_to_graph
from xnn_b200.models.outputs import ForceStressOutput


@pytest.fixture(autouse=True)
def _f64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _butane():
    pos = [[0.0, 0.0, 0.0], [1.53, 0.0, 0.0], [2.05, 1.44, 0.0], [3.58, 1.44, 0.0], [-0.4, -0.5, 0.9],
           [-0.4, -0.5, -0.9], [-0.4, 1.0, 0.0], [1.93, -0.52, 0.88], [1.93, -0.52, -0.88], [1.65, 1.96, -0.88],
           [1.65, 1.96, 0.88], [3.98, 0.44, 0.0], [3.98, 1.96, 0.88], [3.98, 1.96, -0.88]]
    z = [6, 6, 6, 6] + [1] * 10
    types = ["opls_80", "opls_81", "opls_81", "opls_80"] + ["opls_85"] * 10
    bonds = [(0, 1), (1, 2), (2, 3), (0, 4), (0, 5), (0, 6), (1, 7), (1, 8), (2, 9), (2, 10), (3, 11), (3, 12),
             (3, 13)]
    return pos, z, types, bonds


def _ethylene(tilt=12.0):
    d, dh, ang = 1.34, 1.08, math.radians(120.0)
    phi = math.radians(tilt)
    y = dh * math.sin(math.pi - ang)
    pos = [[0.0, 0.0, 0.0], [d, 0.0, 0.0], [-dh * math.cos(math.pi - ang), y, 0], [-dh * math.cos(math.pi - ang), -y, 0],
           [d + dh * math.cos(math.pi - ang), y * math.cos(phi), y * math.sin(phi)],
           [d + dh * math.cos(math.pi - ang), -y, 0.0]]
    return pos, [6, 6, 1, 1, 1, 1], ["opls_88", "opls_88"] + ["opls_89"] * 4, [(0, 1), (0, 2), (0, 3), (1, 4), (1, 5)]


def _graphs(pos, z, cutoff, n=3, cell=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for k in range(n):
        p = torch.tensor(pos) + 0.08 * torch.randn(len(pos), 3, generator=g) * (k > 0)
        s = {"pos": p, "atomic_numbers": torch.tensor(z)}
        if cell is not None:
            s["cell"], s["pbc"] = torch.tensor(cell), torch.tensor([True, True, True])
        out.append(structure_to_graph(s, cutoff))
    return collate(out)


def test_frc_reader_matches_reference():
    rf = ref_module("xnn.ffnn.common.frc")
    from pathlib import Path

    from xnn_b200.ffnn import frc
    for f in ("oplsaa", "lopls", "amber", "charmm22", "dreiding"):
        mine, ref = frc.FrcFile(frc.DATA_DIR / f"{f}.frc"), rf.FrcFile(Path(rf.builtin_data_dir()) / f"{f}.frc")
        assert mine.forcefields == ref.forcefields
        for name in ref.forcefields:
            a, b = mine.forcefield(name), ref.forcefield(name)
            assert set(a.sections) == set(b.sections) and a.metadata == b.metadata
            for kind, rows in b.sections.items():
                assert set(a.sections[kind]) == set(rows)
                for key, row in rows.items():
                    for col, v in row.values.items():
                        w = a.sections[kind][key].values[col]
                        assert (math.isclose(float(w), float(v), rel_tol=1e-12, abs_tol=1e-14)
                                if isinstance(v, float) else str(w) == str(v)), (f, kind, key, col)


def test_units_and_nonbond_forms():
    from xnn_b200.ffnn.frc import convert_units, nonbond_to_sigma_eps
    assert math.isclose(convert_units(1.0, "kJ/mol/nm^2", "kcal/mol/Å^2"), 1.0 / 418.4)
    assert math.isclose(convert_units(2.0, "(kcal/mol)**(1/12)*nm", "(kcal/mol)**(1/12)*Å"), 20.0)
    s, e = nonbond_to_sigma_eps("A-B", 4.0 * 0.2 * 3.0 ** 12, 4.0 * 0.2 * 3.0 ** 6)
    assert math.isclose(s, 3.0) and math.isclose(e, 0.2)
    with pytest.raises(ValueError):
        convert_units(1.0, "kcal/mol", "Å")


def test_topology_derivation_matches_reference():
    rt = ref_module("xnn.ffnn.models.topology")
    from xnn_b200.ffnn.topology import MolecularTopology, guess_bonds
    pos, z, types, bonds = _butane()
    a, b = MolecularTopology.from_bonds(types, bonds), rt.MolecularTopology.from_bonds(types, bonds)
    for f in ("bonds", "angles", "dihedrals", "exclusions", "pairs14", "pairs15"):
        assert getattr(a, f) == getattr(b, f), f
    assert guess_bonds(pos, z) == sorted(bonds) == rt.guess_bonds(pos, z)
    r = a.replicate(3)
    assert r.n_atoms == 42 and r.pairs14[-1] == tuple(x + 28 for x in a.pairs14[-1])


@pytest.mark.parametrize("case", ["butane", "butane_switch", "ethylene", "periodic"])
def test_opls_matches_reference(case):
    ro = ref_module("xnn.ffnn.models.opls")
    rt = ref_module("xnn.ffnn.models.topology")
    from ref_oracle import ref_graph
    from xnn_b200.ffnn.opls import OPLS
    from xnn_b200.ffnn.topology import MolecularTopology
    pos, z, types, bonds = _ethylene() if case == "ethylene" else _butane()
    cell, cutoff, kw = None, 20.0, {}
    if case == "butane_switch":
        cutoff, kw = 4.0, {"switch_width": 1.5}
    if case == "periodic":
        cell, cutoff = [[9.0, 0.0, 0.0], [0.0, 8.5, 0.0], [0.0, 0.0, 9.5]], 4.0
    mine = OPLS("oplsaa", MolecularTopology.from_bonds(types, bonds), cutoff=cutoff, **kw)
    ref = ro.OPLS("oplsaa", rt.MolecularTopology.from_bonds(types, bonds), cutoff=cutoff, use_fast=False, **kw)
    b = _graphs(pos, z, cutoff, cell=cell)
    outs = ref_module("xnn.common.models.outputs")
    periodic = cell is not None
    o_ref = outs.ForceStressOutput(ref, compute_stress=periodic)(ref_graph(b))
    o = ForceStressOutput(mine, compute_stress=periodic)(b.clone())
    for k in ("energy", "forces", "e_bond", "e_angle", "e_torsion", "e_improper", "e_lj", "e_coulomb", "e_lj14",
              "e_coulomb14") + (("stress",) if periodic else ()):
        torch.testing.assert_close(o[k], o_ref[k], rtol=1e-10, atol=1e-10, msg=k)
    assert float(o["e_torsion"].detach().abs().sum()) > 0
    key = "e_improper" if case == "ethylene" else "e_lj"
    assert float(o[key].detach().abs().sum()) > 0


def test_opls_training_keeps_net_charge_and_library_roundtrip(tmp_path):
    from xnn_b200.ffnn.opls import OPLS, read_opls
    from xnn_b200.ffnn.topology import MolecularTopology
    pos, z, types, bonds = _butane()
    m = OPLS("oplsaa", MolecularTopology.from_bonds(types, bonds), cutoff=20.0, trainable=["charge", "bond_k"])
    with torch.no_grad():
        m.ff.params["charge"].add_(0.1)
    q = m(_graphs(pos, z, 20.0, n=1))["charges"]
    assert abs(float(q.detach().sum())) < 1e-10
    lib = m.export_library()
    lib.save(tmp_path / "lib.json")
    back = read_opls(tmp_path / "lib.json")
    e1 = m(_graphs(pos, z, 20.0, n=1))["energy"]
    e2 = OPLS(back, MolecularTopology.from_bonds(types, bonds), cutoff=20.0)(_graphs(pos, z, 20.0, n=1))["energy"]
    torch.testing.assert_close(e1, e2, rtol=1e-9, atol=1e-9)


def _nma():
    pos = [[0.0, 0.0, 0.0], [1.51, 0.0, 0.0], [2.13, 1.07, 0.0], [2.14, -1.19, 0.0], [3.59, -1.28, 0.0],
           [1.60, -2.05, 0.0], [-0.38, 1.02, 0.0], [-0.38, -0.51, 0.89], [-0.38, -0.51, -0.89], [3.95, -0.76, 0.89],
           [3.95, -0.76, -0.89], [3.95, -2.31, 0.0]]
    z = [6, 6, 8, 7, 6, 1, 1, 1, 1, 1, 1, 1]
    types = ["CT", "C", "O", "N", "CT", "H", "HC", "HC", "HC", "H1", "H1", "H1"]
    bonds = [(0, 1), (1, 2), (1, 3), (3, 4), (3, 5), (0, 6), (0, 7), (0, 8), (4, 9), (4, 10), (4, 11)]
    q = [-0.3662, 0.5972, -0.5679, -0.4157, -0.1490, 0.2719, 0.1123, 0.1123, 0.1123, 0.0976, 0.0976, 0.0976]
    return pos, z, types, bonds, q


@pytest.mark.parametrize("periodic", [False, True])
def test_amber_matches_reference(periodic):
    ra = ref_module("xnn.ffnn.models.amber")
    rt = ref_module("xnn.ffnn.models.topology")
    from ref_oracle import ref_graph
    from xnn_b200.ffnn.amber import Amber
    from xnn_b200.ffnn.topology import MolecularTopology
    pos, z, types, bonds, q = _nma()
    cell, cutoff = ([[10.0, 0, 0], [0, 9.0, 0], [0, 0, 9.5]], 4.0) if periodic else (None, 20.0)
    mine = Amber("ff94", MolecularTopology.from_bonds(types, bonds, charges=q), cutoff=cutoff, switch_width=1.0)
    ref = ra.Amber("ff94", rt.MolecularTopology.from_bonds(types, bonds, charges=q), cutoff=cutoff, switch_width=1.0,
                   use_fast=False)
    assert mine.impropers == ref.impropers and len(mine.impropers) == 2
    b = _graphs(pos, z, cutoff, cell=cell)
    outs = ref_module("xnn.common.models.outputs")
    o_ref = outs.ForceStressOutput(ref, compute_stress=periodic)(ref_graph(b))
    o = ForceStressOutput(mine, compute_stress=periodic)(b.clone())
    for k in ("energy", "forces", "e_torsion", "e_improper", "e_vdw", "e_coulomb", "e_vdw14", "e_coulomb14") + \
            (("stress",) if periodic else ()):
        torch.testing.assert_close(o[k], o_ref[k], rtol=1e-10, atol=1e-10, msg=k)
    assert float(o["e_improper"].detach().abs().sum()) > 0


@pytest.mark.parametrize("periodic", [False, True])
def test_charmm_matches_reference(periodic):
    rc = ref_module("xnn.ffnn.models.charmm")
    rt = ref_module("xnn.ffnn.models.topology")
    from ref_oracle import ref_graph
    from xnn_b200.ffnn.charmm import Charmm
    from xnn_b200.ffnn.topology import MolecularTopology
    pos, z, _types, bonds, _q = _nma()
    types = ["CT3", "C", "O", "NH1", "CT3", "H", "HA", "HA", "HA", "HA", "HA", "HA"]
    q = [-0.27, 0.51, -0.51, -0.47, -0.11, 0.31, 0.09, 0.09, 0.09, 0.09, 0.09, 0.09]
    imps = [(1, 0, 3, 2), (3, 1, 4, 5)]
    cell, cutoff = ([[10.0, 0, 0], [0, 9.0, 0], [0, 0, 9.5]], 4.0) if periodic else (None, 20.0)
    mine = Charmm("charmm22", MolecularTopology.from_bonds(types, bonds, charges=q, impropers=imps), cutoff=cutoff,
                  switch_width=1.0)
    ref = rc.Charmm("charmm22", rt.MolecularTopology.from_bonds(types, bonds, charges=q, impropers=imps),
                    cutoff=cutoff, switch_width=1.0, use_fast=False)
    b = _graphs(pos, z, cutoff, cell=cell)
    outs = ref_module("xnn.common.models.outputs")
    o_ref = outs.ForceStressOutput(ref, compute_stress=periodic)(ref_graph(b))
    o = ForceStressOutput(mine, compute_stress=periodic)(b.clone())
    for k in ("energy", "forces", "e_urey_bradley", "e_torsion", "e_improper", "e_vdw", "e_coulomb", "e_vdw14",
              "e_coulomb14") + (("stress",) if periodic else ()):
        torch.testing.assert_close(o[k], o_ref[k], rtol=1e-10, atol=1e-10, msg=k)
    assert float(o["e_improper"].detach().abs().sum()) > 0 and float(o["e_urey_bradley"].detach().abs().sum()) > 0


def _water_dimer():
    pos = [[0.0, 0.0, 0.0], [0.96, 0.0, 0.0], [-0.24, 0.93, 0.0], [2.9, 0.1, 0.2], [3.2, 0.9, 0.5], [3.3, -0.6, 0.6]]
    return pos, [8, 1, 1, 8, 1, 1], ["O_3", "H__HB", "H__HB", "O_3", "H__HB", "H__HB"], [(0, 1), (0, 2), (3, 4), (3, 5)]


def _propene():
    pos = [[0.0, 0.0, 0.0], [1.34, 0.0, 0.0], [2.1, 1.3, 0.0], [-0.55, 0.93, 0.0], [-0.55, -0.93, 0.0],
           [1.9, -0.93, 0.0], [3.15, 1.05, 0.1], [1.85, 1.9, 0.88], [1.9, 1.92, -0.85]]
    return (pos, [6, 6, 6, 1, 1, 1, 1, 1, 1], ["C_2", "C_2", "C_3"] + ["H_"] * 6,
            [(0, 1), (1, 2), (0, 3), (0, 4), (1, 5), (2, 6), (2, 7), (2, 8)])


@pytest.mark.parametrize("case", ["propene", "propene_x6_morse", "water", "water_periodic"])
def test_dreiding_matches_reference(case):
    rd = ref_module("xnn.ffnn.models.dreiding")
    rt = ref_module("xnn.ffnn.models.topology")
    from ref_oracle import ref_graph
    from xnn_b200.ffnn.dreiding import Dreiding
    from xnn_b200.ffnn.topology import MolecularTopology
    if case.startswith("water"):
        pos, z, types, bonds = _water_dimer()
        orders, q = [1.0] * 4, [-0.8, 0.4, 0.4, -0.8, 0.4, 0.4]
    else:
        pos, z, types, bonds = _propene()
        orders, q = [2.0] + [1.0] * 7, None
    kw = dict(bond_style="morse", angle_style="harmonic") if case == "propene_x6_morse" else {}
    ffield = "dreiding/X6" if case == "propene_x6_morse" else "dreiding"
    cell, cutoff = ([[8.0, 0, 0], [0, 7.5, 0], [0, 0, 7.0]], 3.5) if case == "water_periodic" else (None, 12.0)
    mine = Dreiding(ffield, MolecularTopology.from_bonds(types, bonds, bond_orders=orders), cutoff=cutoff, charges=q, **kw)
    ref = rd.Dreiding(ffield, rt.MolecularTopology.from_bonds(types, bonds, bond_orders=orders), cutoff=cutoff,
                      charges=q, use_fast=False, **kw)
    b = _graphs(pos, z, cutoff, cell=cell)
    periodic = cell is not None
    outs = ref_module("xnn.common.models.outputs")
    o_ref = outs.ForceStressOutput(ref, compute_stress=periodic)(ref_graph(b))
    o = ForceStressOutput(mine, compute_stress=periodic)(b.clone())
    for k in ("energy", "forces", "e_bond", "e_angle", "e_torsion", "e_inversion", "e_vdw", "e_coulomb", "e_hbond") \
            + (("stress",) if periodic else ()):
        torch.testing.assert_close(o[k], o_ref[k], rtol=1e-10, atol=1e-10, msg=k)
    key = "e_hbond" if case.startswith("water") else "e_torsion"
    assert float(o[key].detach().abs().sum()) > 0


@pytest.mark.parametrize("kind", ["opls", "amber"])
def test_lammps_input_matches_reference(kind, tmp_path):
    rl = ref_module("xnn.ffnn.models.lammps_input")
    rt = ref_module("xnn.ffnn.models.topology")
    from xnn_b200.ffnn.lammps_input import lammps_input, write_lammps_input
    from xnn_b200.ffnn.topology import MolecularTopology
    if kind == "opls":
        ro = ref_module("xnn.ffnn.models.opls")
        from xnn_b200.ffnn.opls import OPLS
        pos, z, types, bonds = _butane()
        mine = OPLS("oplsaa", MolecularTopology.from_bonds(types, bonds), cutoff=9.0)
        ref = ro.OPLS("oplsaa", rt.MolecularTopology.from_bonds(types, bonds), cutoff=9.0, use_fast=False)
        cell = None
    else:
        ra = ref_module("xnn.ffnn.models.amber")
        from xnn_b200.ffnn.amber import Amber
        pos, z, types, bonds, q = _nma()
        mine = Amber("ff94", MolecularTopology.from_bonds(types, bonds, charges=q), cutoff=4.0)
        ref = ra.Amber("ff94", rt.MolecularTopology.from_bonds(types, bonds, charges=q), cutoff=4.0, use_fast=False)
        cell = [[10.0, 0, 0], [0, 9.0, 0], [0, 0, 9.5]]
    data, cmds, off = lammps_input(mine, torch.tensor(pos), cell)
    rdata, rcmds, roff, _files = rl.lammps_input(ref, torch.tensor(pos), cell)
    assert data == rdata and cmds == rcmds and off == roff
    assert write_lammps_input(mine, torch.tensor(pos), cell, tmp_path).read_text().count("_coeff") > 5


@pytest.mark.parametrize("case", ["charmm", "dreiding_water", "dreiding_x6_morse"])
def test_lammps_input_charmm_dreiding(case, tmp_path):
    rl = ref_module("xnn.ffnn.models.lammps_input")
    rt = ref_module("xnn.ffnn.models.topology")
    from xnn_b200.ffnn.lammps_input import lammps_input, write_lammps_input
    from xnn_b200.ffnn.topology import MolecularTopology
    if case == "charmm":
        rc = ref_module("xnn.ffnn.models.charmm")
        from xnn_b200.ffnn.charmm import Charmm
        pos, z, _types, bonds, _q = _nma()
        types = ["CT3", "C", "O", "NH1", "CT3", "H", "HA", "HA", "HA", "HA", "HA", "HA"]
        q = [-0.27, 0.51, -0.51, -0.47, -0.11, 0.31, 0.09, 0.09, 0.09, 0.09, 0.09, 0.09]
        imps = [(1, 0, 3, 2), (3, 1, 4, 5)]
        mine = Charmm("charmm22", MolecularTopology.from_bonds(types, bonds, charges=q, impropers=imps), cutoff=8.0)
        ref = rc.Charmm("charmm22", rt.MolecularTopology.from_bonds(types, bonds, charges=q, impropers=imps),
                        cutoff=8.0, use_fast=False)
        cell = None
    else:
        rd = ref_module("xnn.ffnn.models.dreiding")
        from xnn_b200.ffnn.dreiding import Dreiding
        if case == "dreiding_water":
            pos, z, types, bonds = _water_dimer()
            orders, q, kw, ffield = [1.0] * 4, [-0.8, 0.4, 0.4, -0.8, 0.4, 0.4], {}, "dreiding"
            cell = [[8.0, 0, 0], [0, 7.5, 0], [0, 0, 7.0]]
        else:
            pos, z, types, bonds = _propene()
            orders, q, ffield = [2.0] + [1.0] * 7, None, "dreiding/X6"
            kw, cell = dict(bond_style="morse", angle_style="harmonic"), None
        mine = Dreiding(ffield, MolecularTopology.from_bonds(types, bonds, bond_orders=orders), cutoff=3.5, charges=q,
                        **kw)
        ref = rd.Dreiding(ffield, rt.MolecularTopology.from_bonds(types, bonds, bond_orders=orders), cutoff=3.5,
                          charges=q, use_fast=False, **kw)
    data, cmds, off = lammps_input(mine, torch.tensor(pos), cell)
    rdata, rcmds, roff, _files = rl.lammps_input(ref, torch.tensor(pos), cell)
    assert data == rdata and cmds == rcmds and off == roff
    assert write_lammps_input(mine, torch.tensor(pos), cell, tmp_path).read_text().count("_coeff") > 3
