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
