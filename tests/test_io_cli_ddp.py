"""Structure files, the command line, and config-1 data-parallel training on Gloo ranks."""
import json
import os

import pytest
import torch

from xnn_b200.data import synthetic
from xnn_b200.data.io import read_extxyz, read_runner, read_structures, write_extxyz, write_runner

from dist_util import run_ranks


def _close(a, b):
    torch.testing.assert_close(torch.as_tensor(a).double(), torch.as_tensor(b).double(), rtol=1e-9, atol=1e-9)


def test_extxyz_and_runner_round_trip(tmp_path):
    mols = synthetic.organic_molecules(3, seed=1)
    crys = synthetic.triclinic_crystals(2, seed=2)
    for s in crys:
        s["stress"] = torch.randn(3, 3, dtype=torch.float64)
        s["stress"] = 0.5 * (s["stress"] + s["stress"].T)
    items = mols + crys
    for write, read, name in ((write_extxyz, read_extxyz, "a.extxyz"), (write_runner, read_runner, "input.data")):
        path = write(items, tmp_path / name)
        back = read(path)
        assert len(back) == len(items)
        for s, b in zip(items, back):
            _close(s["pos"], b["pos"])
            assert torch.equal(torch.as_tensor(s["atomic_numbers"]), b["atomic_numbers"])
            assert abs(float(s["energy"]) - float(b["energy"])) < 1e-8
            _close(s["forces"], b["forces"])
            if s.get("cell") is not None:
                _close(s["cell"], b["cell"])
        assert read_structures(path)[0]["pos"].shape == items[0]["pos"].shape


def _train_cfg(tmp_path, extra=None):
    return ["--set", "model.name=nequip", "--set", "model.cutoff=5.0", "--set", "model.n_features=8",
            "--set", "model.n_interactions=2", "--set", "model.n_rbf=8", "--set", "model.extra.l_max=1",
            "--set", "model.extra.species=[1,6,8]",
            "--set", "data.train_path=synthetic:small:20", "--set", "data.batch_size=5",
            "--set", "data.val_fraction=0.2", "--set", "optim.epochs=2", "--set", "optim.force_weight=100.0",
            "--set", "device=cpu", "--set", f"output_dir={tmp_path}", "--set", "trainer.loggers=[]"] + (extra or [])


def test_cli_train_benchmark_export(tmp_path, capsys):
    from xnn_b200.cli import main
    assert main(["train"] + _train_cfg(tmp_path)) == 0
    assert os.path.exists(tmp_path / "best.pt") and os.path.exists(tmp_path / "last.pt")
    data = write_extxyz(synthetic.small_organic(4, seed=9), tmp_path / "test.extxyz")
    capsys.readouterr()
    assert main(["benchmark", "--model", str(tmp_path / "best.pt"), "--data", str(data), "--format", "json"]) == 0
    report = json.loads(capsys.readouterr().out)
    assert report["forces"]["n"] == 4 * 21 * 3 and report["energy"]["mae"] >= 0
    assert main(["export", "--model", str(tmp_path / "best.pt"), "--format", "lammps",
                 "--out", str(tmp_path / "m.pt")]) == 0
    assert os.path.exists(tmp_path / "m.pt")


def _ddp_rank(rank, world, out_dir):
    from xnn_b200.cli.main import build_parser
    from xnn_b200.config import from_argparse
    from xnn_b200.data import AtomicDataset
    from xnn_b200.train import Trainer
    args = build_parser().parse_args(["train"] + _train_cfg(out_dir))
    cfg = from_argparse(args)
    ds = AtomicDataset(synthetic.small_organic(20, seed=cfg.seed), float(cfg.model.cutoff))
    tr = Trainer(cfg, ds)
    tr.fit()
    flat = torch.cat([p.detach().reshape(-1) for p in tr.module.parameters()])
    tr.close()
    return flat


def test_gloo_two_rank_training_keeps_replicas_identical(tmp_path):
    a, b = run_ranks(_ddp_rank, 2, str(tmp_path))
    assert torch.equal(a, b)
    assert os.path.exists(tmp_path / "best.pt")


def _mace_engine_rank(rank, world, out_dir):
    from xnn_b200.config import from_dict
    from xnn_b200.data import AtomicDataset
    from xnn_b200.train import Trainer
    torch.set_default_dtype(torch.float64)
    cfg = from_dict({
        "model": {"name": "mace", "cutoff": 4.5, "n_features": 8, "n_interactions": 2, "n_rbf": 6,
                  "extra": {"species": [1, 6, 8], "max_ell": 2, "correlation": 2, "avg_num_neighbors": 8.0}},
        "optim": {"lr": 1e-3, "epochs": 2, "force_weight": 10.0, "scheduler": "none"},
        "data": {"batch_size": 3, "val_fraction": 0.0},
        "trainer": {"loggers": [], "fused_step": True},
        "device": "cpu", "seed": 5, "output_dir": str(out_dir)})
    ds = AtomicDataset(synthetic.small_organic(12, seed=cfg.seed), 4.5)
    tr = Trainer(cfg, ds, val=[], test=[])
    assert tr._fused is not None and tr.grad_sync.n_buckets == 3
    tr.fit()
    flat = torch.cat([p.detach().reshape(-1) for p in tr.module.parameters()])
    tr.close()
    return flat


def test_gloo_two_rank_engine_with_gradient_buckets(tmp_path):
    """The hand-written MACE step with per-interaction gradient buckets reduced as they finish:
    both replicas stay identical."""
    a, b = run_ranks(_mace_engine_rank, 2, str(tmp_path))
    assert torch.equal(a, b)
