"""Learned loss-term weights (optim.loss_weighting: uncertainty): the objective's closed form, the
trainer learning log sigma per active term, and the checkpoint recording the sigmas."""
import math

import pytest
import torch

from xnn_b200.config import from_dict
from xnn_b200.data import AtomicDataset, synthetic
from xnn_b200.train import Trainer
from xnn_b200.train.losses import UncertaintyWeights


def test_objective_closed_form():
    uw = UncertaintyWeights(["energy_mse", "force_mse"])
    with torch.no_grad():
        uw.log_sigma["energy_mse"].fill_(0.3)
        uw.log_sigma["force_mse"].fill_(-0.2)
    parts = {"energy_mse": torch.tensor(2.0), "force_mse": torch.tensor(5.0), "stress_mse": torch.tensor(1.5)}
    want = 0.5 * math.exp(-0.6) * 2.0 + 0.3 + 0.5 * math.exp(0.4) * 5.0 - 0.2 + 1.5
    assert abs(float(uw(parts)) - want) < 1e-6
    assert abs(uw.sigmas()["energy_mse"] - math.exp(0.3)) < 1e-6


def _cfg(tmp_path, weighting, graph=False):
    return from_dict({"model": {"name": "schnet", "cutoff": 4.0, "n_features": 16, "n_interactions": 1, "n_rbf": 8},
                      "optim": {"lr": 5e-2, "energy_weight": 1.0, "force_weight": 10.0, "epochs": 2,
                                "scheduler": "none", "loss_weighting": weighting},
                      "data": {"batch_size": 4, "val_fraction": 0.0},
                      "trainer": {"loggers": [], "cuda_graph": graph},
                      "device": "cpu", "seed": 3, "output_dir": str(tmp_path)})


def test_trainer_learns_sigmas_and_saves_them(tmp_path):
    ds = AtomicDataset(synthetic.small_organic(8, seed=2), 4.0)
    tr = Trainer(_cfg(tmp_path, "uncertainty"), ds, val=[], test=[])
    assert set(tr.loss_weights.log_sigma) == {"energy_mse", "force_mse"}
    before = {k: float(v) for k, v in tr.loss_weights.log_sigma.items()}
    tr.fit()
    after = {k: float(v) for k, v in tr.loss_weights.log_sigma.items()}
    assert any(abs(after[k] - before[k]) > 1e-4 for k in before)
    path = str(tmp_path / "ck.pt")
    tr.save(path)
    state = torch.load(path, weights_only=False)
    assert set(state["loss_sigmas"]) == {"energy_mse", "force_mse"}


def test_rejected_settings(tmp_path):
    ds = AtomicDataset(synthetic.small_organic(4, seed=2), 4.0)
    with pytest.raises(ValueError, match="loss_weighting"):
        Trainer(_cfg(tmp_path, "learned"), ds, val=[], test=[])


def test_hydra_and_override_loaders():
    from collections import OrderedDict

    from xnn_b200.config import apply_overrides, from_hydra

    class Node(OrderedDict):          # a mapping standing in for an OmegaConf DictConfig
        pass

    node = Node(model=Node(name="schnet", cutoff=4.5, n_features=32), optim=Node(lr=0.002, loss_weighting="uncertainty"))
    cfg = from_hydra(node)
    assert cfg.model.name == "schnet" and cfg.model.cutoff == 4.5 and cfg.optim.loss_weighting == "uncertainty"
    cfg2 = apply_overrides(cfg, ["model.cutoff=6.0", "optim.lr=1e-3"])
    assert cfg2.model.cutoff == 6.0 and cfg2.data.cutoff == 6.0 and abs(cfg2.optim.lr - 1e-3) < 1e-12
