"""Benchmark suites on the CPU: selection by label / shard, part files and their merge, and the
one-worker-per-model fan-out through the command line."""
import json
import os

import pytest
import torch
import yaml

from xnn_b200.benchmark import suite as S
from xnn_b200.config import from_dict
from xnn_b200.data import synthetic
from xnn_b200.data.io import write_extxyz
from xnn_b200.hub import save_pretrained
from xnn_b200.models.registry import prepare_model


@pytest.fixture()
def suite_file(tmp_path):
    models = []
    for k, name in enumerate(["schnet", "painn", "schnet"]):
        cfg = from_dict({"model": {"name": name, "cutoff": 4.0, "n_features": 8, "n_interactions": 1, "n_rbf": 6},
                         "device": "cpu", "seed": k})
        torch.manual_seed(k)
        d = save_pretrained(prepare_model(cfg), tmp_path / f"m{k}", config=cfg)
        models.append({"label": f"{name}-{k}", "model": str(d)})
    data = write_extxyz(synthetic.small_organic(6, seed=3), tmp_path / "data.extxyz")
    path = tmp_path / "suite.yaml"
    path.write_text(yaml.safe_dump({"models": models, "data": str(data), "batch_size": 4, "device": "cpu",
                                    "output": {"dir": str(tmp_path / "out"), "filename": "res",
                                               "formats": ["json", "md"]}}))
    return str(path)


def test_selection_and_shards(suite_file):
    cfg = S.load_suite(suite_file)
    assert [e["label"] for e in S.select_entries(cfg, "painn-1,0")] == ["painn-1", "schnet-0"]
    shards = [S.select_entries(cfg, shard=f"{i}/2") for i in range(2)]
    assert sorted(e["label"] for s in shards for e in s) == sorted(e["label"] for e in cfg["models"])
    with pytest.raises(ValueError):
        S.select_entries(cfg, "nope")
    with pytest.raises(ValueError):
        S.select_entries(cfg, shard="3/2")


def test_parts_merge_and_parallel(suite_file):
    cfg = S.load_suite(suite_file)
    for i in range(2):
        ent = S.select_entries(cfg, shard=f"{i}/2")
        S.write_part(cfg, S.score(cfg, ent), ent)
    rows = S.merge_parts(cfg)
    assert [r["model"] for r in rows] == [e["label"] for e in cfg["models"]]
    assert all(r["energy_n"] == 6 and r["forces_mae"] > 0 for r in rows)
    assert os.path.exists(os.path.join(cfg["output"]["dir"], "res.md"))
    # the same table from one worker process per model (two at a time)
    for f in os.listdir(os.path.join(cfg["output"]["dir"], "parts")):
        os.remove(os.path.join(cfg["output"]["dir"], "parts", f))
    rows2 = S.run_parallel(suite_file, workers=2)
    for a, b in zip(rows, rows2):
        assert a["model"] == b["model"] and abs(a["energy_mae"] - b["energy_mae"]) < 1e-9
    with open(os.path.join(cfg["output"]["dir"], "res.json")) as f:
        assert len(json.load(f)) == 3
