"""Dataset hub: registry, offline behaviour, rMD17 / QM7 readers on stand-in files with the
published layouts, the synthetic sets and the file builder."""
import numpy as np
import pytest

from xnn_b200.data.hub import list_datasets, load_dataset
from xnn_b200.data.hub import download


def test_registry_lists_builders():
    assert {"rmd17", "qm7", "argon_md", "file", "synthetic"} <= set(list_datasets())
    with pytest.raises(KeyError):
        load_dataset("nope")


def test_offline_missing_file_names_the_path(tmp_path, monkeypatch):
    monkeypatch.setenv("XNN_B200_OFFLINE", "1")
    with pytest.raises(FileNotFoundError, match="rmd17_ethanol.npz"):
        load_dataset("rmd17", molecule="ethanol", cache_dir=tmp_path)


def test_rmd17_reader_units_and_splits(tmp_path, monkeypatch):
    monkeypatch.setenv("XNN_B200_OFFLINE", "1")
    monkeypatch.setattr(download, "md5sum", lambda p: None)      # stand-in files: no published checksums
    import xnn_b200.data.hub.builders as B
    monkeypatch.setattr(B, "_RMD17", {k: (v[0], None) for k, v in B._RMD17.items()})
    monkeypatch.setattr(B, "_RMD17_SPLITS", {k: (v[0], None) for k, v in B._RMD17_SPLITS.items()})
    raw = tmp_path / "rmd17" / "raw"
    raw.mkdir(parents=True)
    rng = np.random.default_rng(0)
    np.savez(raw / "rmd17_ethanol.npz", nuclear_charges=np.array([6, 6, 8, 1, 1, 1, 1, 1, 1]),
             coords=rng.normal(size=(10, 9, 3)), energies=rng.normal(size=10) * 100, forces=rng.normal(size=(10, 9, 3)))
    np.savetxt(raw / "index_train_01.csv", np.arange(7), fmt="%d")
    np.savetxt(raw / "index_test_01.csv", np.arange(7, 10), fmt="%d")
    d = load_dataset("rmd17", molecule="Ethanol", cache_dir=tmp_path)
    assert len(d["train"]) == 7 and len(d["test"]) == 3
    e = np.load(raw / "rmd17_ethanol.npz")["energies"]
    assert abs(d["train"][0]["energy"] - e[0] * 0.0433641153087705) < 1e-9
    kcal = load_dataset("rmd17", molecule="ethanol", units="kcal/mol", split="all", cache_dir=tmp_path)
    assert len(kcal) == 10 and abs(kcal[3]["energy"] - e[3]) < 1e-9
    ds = load_dataset("rmd17", molecule="ethanol", split="test", cutoff=4.0, cache_dir=tmp_path)
    assert len(ds) == 3


def test_qm7_reader(tmp_path, monkeypatch):
    from scipy.io import savemat
    monkeypatch.setenv("XNN_B200_OFFLINE", "1")
    import xnn_b200.data.hub.builders as B
    monkeypatch.setattr(B, "_QM7", (B._QM7[0], None))
    raw = tmp_path / "qm7" / "raw"
    raw.mkdir(parents=True)
    rng = np.random.default_rng(1)
    Z = np.zeros((10, 23))
    Z[:, :5] = [6, 1, 1, 1, 1]
    savemat(raw / "qm7.mat", {"R": rng.normal(size=(10, 23, 3)), "Z": Z, "T": rng.normal(size=(1, 10)),
                              "P": np.arange(10).reshape(5, 2)})
    d = load_dataset("qm7", cache_dir=tmp_path, fold=2)
    assert len(d["train"]) == 8 and len(d["test"]) == 2
    assert d["test"][0]["atomic_numbers"].tolist() == [6, 1, 1, 1, 1]


def test_synthetic_and_file_builders(tmp_path):
    from xnn_b200.data.io import write_extxyz
    items = load_dataset("synthetic", kind="organic", n=5, seed=3)
    assert len(items) == 5 and "forces" in items[0]
    path = tmp_path / "x.extxyz"
    write_extxyz(items, str(path))
    back = load_dataset("file", path=str(path))
    assert len(back) == 5
    np.testing.assert_allclose(np.asarray(back[2]["pos"]), np.asarray(items[2]["pos"]), atol=1e-6)


def _qm9_xyz(index, symbols, coords, props):
    lines = [f"{len(symbols)}", "gdb " + str(index) + "\t" + "\t".join(repr(p) for p in props)]
    lines += [f"{s}\t" + "\t".join(c) + "\t0.0" for s, c in zip(symbols, coords)]
    return "\n".join(lines + ["freq", "SMILES", "InChI"]) + "\n"


def test_qm9_reader(tmp_path, monkeypatch):
    import io
    import tarfile

    from xnn_b200.data.hub import qm9
    root = tmp_path / "qm9" / "raw"
    root.mkdir(parents=True)
    props = [[1.0 * k + p for p in range(15)] for k in range(4)]
    mols = {1: (["C", "H", "H", "H", "H"], [["0.0", "0.0", "0.0"], ["1.09", "0", "0"], ["-0.36", "1.03", "0"],
                                            ["-0.36", "-0.5", "0.9"], ["-0.36", "-0.5", "-0.9"]]),
            2: (["O", "H", "H"], [["0", "0", "0"], ["0.96", "0", "0"], ["-2.4*^-1", "0.93", "0"]]),
            3: (["N", "H", "H", "H"], [["0", "0", "0"], ["1.0", "0", "0"], ["0", "1.0", "0"], ["0", "0", "1.0"]]),
            4: (["F", "H"], [["0", "0", "0"], ["0.92", "0", "0"]])}
    with tarfile.open(root / "dsgdb9nsd.xyz.tar.bz2", "w:bz2") as tar:
        for k in (3, 1, 4, 2):                     # archive order is not index order
            data = _qm9_xyz(k, *mols[k], props[k - 1]).encode()
            info = tarfile.TarInfo(f"dsgdb9nsd_{k:06d}.xyz")
            info.size = len(data)
            tar.addfile(info, io.BytesIO(data))
    (root / "uncharacterized.txt").write_text("header\n   4   x\n")
    monkeypatch.setattr(qm9, "XYZ_ARCHIVE", (qm9.XYZ_ARCHIVE[0], None))
    monkeypatch.setattr(qm9, "UNCHARACTERIZED", (qm9.UNCHARACTERIZED[0], None))
    monkeypatch.setenv("XNN_B200_OFFLINE", "1")
    every = load_dataset("qm9", split="all", cache_dir=tmp_path, return_info=True)
    assert [s["info"]["index"] for s in every] == [1, 2, 3]          # molecule 4 is uncharacterized
    assert every[1]["atomic_numbers"].tolist() == [8, 1, 1] and abs(every[1]["pos"][2, 0] + 0.24) < 1e-12
    hartree = 27.211386245988
    assert abs(every[0]["energy"] - (0 + 10) * hartree) < 1e-9       # U0 column, eV
    assert abs(every[0]["info"]["mu"] - 3.0) < 1e-12                 # not an energy: unscaled
    s = load_dataset("qm9", cache_dir=tmp_path, n_train=2, n_val=1, label="gap", units="hartree")
    assert [len(s[k]) for k in ("train", "val", "test")] == [2, 1, 0]
    assert abs(qm9.atomic_energies("U0")[1] + 0.500273 * hartree) < 1e-9


def test_gmtkn55_reader(tmp_path, monkeypatch):
    import zipfile

    from xnn_b200.data.hub import gmtkn55
    from xnn_b200.train.reactions import ReactionSet
    arc = tmp_path / "gmtkn55" / "raw" / "GMTKN55-v2.zip"
    arc.parent.mkdir(parents=True)
    top = "GMTKN55-commit/"
    files = {"W4-11/.res": "# comment\n$tmer h2 h x -1 2 $w 109.49\n$tmer h2o h2 o x -1 1 1 $w 232.97 0 1\n",
             "W4-11/h2/struc.xyz": "2\n\nH 0 0 0\nH 0 0 0.74\n",
             "W4-11/h/struc.xyz": "1\n\nH 0 0 0\n", "W4-11/h/.UHF": "1\n",
             "W4-11/o/struc.xyz": "1\n\nO 0 0 0\n", "W4-11/o/.UHF": "2\n",
             "W4-11/h2o/struc.xyz": "3\n\nO 0 0 0\nH 0.96 0 0\nH -0.24 0.93 0\n",
             "BH76/.resRC": "$tmer h{2,2o} x 1 -1 $w 1.5\n",
             "BH76/h2o/struc.xyz": "3\n\nO 0 0 0\nH 0.96 0 0\nH -0.24 0.93 0\n",
             "BH76/h2/struc.xyz": "2\n\nH 0 0 0\nH 0 0 0.74\n", "BH76/h2/.CHRG": "0\n",
             "W4-11/h2o/PBEh-3c/orca.out": "FINAL SINGLE POINT ENERGY   -76.25\n"}
    with zipfile.ZipFile(arc, "w") as zf:
        for name, text in files.items():
            zf.writestr(top + name, text)
    monkeypatch.setattr(gmtkn55, "VERSIONS", {"v2": ("commit", None)})
    monkeypatch.setenv("XNN_B200_OFFLINE", "1")
    data = load_dataset("gmtkn55", cache_dir=tmp_path, subsets=["w4-11", "BH76RC"])
    assert [r["species"] for r in data["reactions"]] == [["h2", "h"], ["h2o", "h2", "o"], ["h2", "h2o"]]
    assert data["reactions"][2]["subset"] == "BH76RC" and data["reactions"][1]["reference"] == 232.97
    w = {(s["subset"], s["name"]): s for s in data["structures"]}
    assert w[("W4-11", "o")]["spin_multiplicity"] == 3.0 and abs(w[("W4-11", "h2o")]["pbeh3c_energy"] + 76.25 * 27.211386245988) < 1e-6
    closed = load_dataset("gmtkn55", cache_dir=tmp_path, subsets="W4-11", closed_shell=True, split="reactions")
    assert closed == []                                                  # both need an open-shell atom
    rs = ReactionSet.from_gmtkn55(data)
    assert len(rs) == 3 and rs.stoichiometry().shape == (3, len(data["structures"]))
