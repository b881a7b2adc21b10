"""OC20 S2EF, Materials Project 2018 and ASE-database builders on stand-in files of the same formats."""
import io
import json
import lzma
import math
import sqlite3
import tarfile
import zipfile

import numpy as np
import pytest
import torch

from xnn_b200.data.hub import list_datasets, load_dataset
from xnn_b200.data.hub.more import parse_p1_cif, read_ase_db

FRAME = """3
Lattice="10.0 0.0 0.0 0.0 10.0 0.0 0.0 0.0 30.0" Properties=species:S:1:pos:R:3:move_mask:L:1:tags:I:1:forces:R:3 energy=-12.5 pbc="T T T"
Pt 0.0 0.0 0.0 F 0 0.0 0.0 0.0
Pt 2.0 0.0 0.0 T 1 0.1 0.0 0.0
O 1.0 1.0 2.0 T 2 -0.1 0.2 0.3
"""


def _oc20(tmp_path):
    path = tmp_path / "s2ef.tar"
    with tarfile.open(path, "w") as tar:
        for name, data in (("s2ef/0.extxyz.xz", lzma.compress((FRAME + FRAME.replace("-12.5", "-11.0")).encode())),
                           ("s2ef/0.txt", b"random1,frame0,-10.0\nrandom1,frame1,-10.0\n")):
            info = tarfile.TarInfo(name)
            info.size = len(data)
            tar.addfile(info, io.BytesIO(data))
    return path


def test_registered():
    assert {"oc20_s2ef_200k", "mp_2018", "ase_db"} <= set(list_datasets())


def test_oc20_adsorption_energies_and_fixed_atoms(tmp_path):
    frames = load_dataset("oc20_s2ef_200k", archive=str(_oc20(tmp_path)), split=None)
    allf = [s for part in frames.values() for s in part]
    assert len(allf) == 2
    e = sorted(s["energy"] for s in allf)
    assert e == pytest.approx([-2.5, -1.0])
    s = allf[0]
    assert s["atom_force_weight"].tolist() == [0.0, 1.0, 1.0]
    assert s["info"]["tags"].tolist() == [0, 1, 2] and s["info"]["system_id"] == "random1"
    assert torch.allclose(s["forces"][2], torch.tensor([-0.1, 0.2, 0.3], dtype=torch.float64))
    total = load_dataset("oc20_s2ef_200k", archive=str(_oc20(tmp_path)), energy="total", split="all")
    assert sorted(s["energy"] for s in total) == pytest.approx([-12.5, -11.0])


CIF = """# generated using pymatgen
data_NaCl
_symmetry_space_group_name_H-M   'P 1'
_cell_length_a   4.0
_cell_length_b   4.0
_cell_length_c   4.0
_cell_angle_alpha   90.0
_cell_angle_beta   90.0
_cell_angle_gamma   60.0
_symmetry_Int_Tables_number   1
loop_
 _symmetry_equiv_pos_site_id
 _symmetry_equiv_pos_as_xyz
  1  'x, y, z'
loop_
 _atom_site_type_symbol
 _atom_site_label
 _atom_site_symmetry_multiplicity
 _atom_site_fract_x
 _atom_site_fract_y
 _atom_site_fract_z
 _atom_site_occupancy
  Na  Na0  1  0.0  0.0  0.0  1
  Cl  Cl1  1  0.5  0.5  0.5  1
"""


def test_p1_cif_and_mp2018(tmp_path):
    s = parse_p1_cif(CIF)
    assert s["atomic_numbers"].tolist() == [11, 17]
    cell = s["cell"]
    assert float(torch.linalg.norm(cell[1])) == pytest.approx(4.0)
    assert float(torch.dot(cell[0], cell[1]) / 16.0) == pytest.approx(math.cos(math.radians(60.0)))
    assert torch.allclose(s["pos"][1], 0.5 * cell.sum(0))
    path = tmp_path / "mp.json.zip"
    entries = [{"material_id": f"mp-{k}", "structure": CIF, "formation_energy_per_atom": -1.5 - k, "band_gap": 5.0,
                "K": 1.3 if k == 0 else None, "G": None} for k in range(10)]
    with zipfile.ZipFile(path, "w") as z:
        z.writestr("mp.2018.6.1.json", json.dumps(entries))
    parts = load_dataset("mp_2018", archive=str(path))
    assert sum(len(v) for v in parts.values()) == 10 and len(parts["train"]) == 8
    one = [s for v in parts.values() for s in v if s["info"]["material_id"] == "mp-0"][0]
    assert one["energy"] == pytest.approx(-3.0) and one["log10_bulk_modulus"] == pytest.approx(1.3)
    assert math.isnan(one["log10_shear_modulus"])


def test_ase_sqlite_database(tmp_path):
    path = tmp_path / "db.db"
    con = sqlite3.connect(path)
    con.execute("CREATE TABLE systems (id INTEGER PRIMARY KEY, numbers BLOB, positions BLOB, cell BLOB, pbc INTEGER, "
                "energy REAL, forces BLOB, stress BLOB, charges BLOB, initial_charges BLOB, key_value_pairs TEXT)")
    pos = np.arange(9, dtype=np.float64).reshape(3, 3)
    con.execute("INSERT INTO systems VALUES (1, ?, ?, ?, 7, -3.25, ?, ?, NULL, NULL, ?)",
                (np.array([8, 1, 1], dtype=np.int32).tobytes(), pos.tobytes(), (5.0 * np.eye(3)).tobytes(),
                 (0.1 * pos).tobytes(), np.arange(6, dtype=np.float64).tobytes(), json.dumps({"tag": "w"})))
    con.execute("INSERT INTO systems VALUES (2, ?, ?, ?, 0, NULL, NULL, NULL, NULL, NULL, NULL)",
                (np.array([6], dtype=np.int32).tobytes(), np.zeros(3).tobytes(), np.zeros(9).tobytes()))
    con.commit()
    con.close()
    rows = read_ase_db(path)
    assert len(rows) == 2 and rows[0]["atomic_numbers"].tolist() == [8, 1, 1]
    assert rows[0]["energy"] == -3.25 and rows[0]["pbc"].tolist() == [True, True, True]
    assert rows[0]["stress"][0, 1] == 5.0 and rows[0]["info"]["tag"] == "w"
    assert "cell" not in rows[1] and "energy" not in rows[1]
    assert len(load_dataset("ase_db", path=str(path), selection="energy IS NOT NULL")) == 1
