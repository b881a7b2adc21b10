"""The shipped configs/ tree: every family file builds its model, and the run config composes its
model and data groups."""
import glob
import os

import pytest
import yaml

from xnn_b200.config import from_dict, from_yaml
from xnn_b200.models.registry import prepare_model

ROOT = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "configs")
FILES = sorted(glob.glob(os.path.join(ROOT, "model", "*.yaml")))


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(p) for p in FILES])
def test_family_file_builds(path):
    with open(path) as f:
        body = yaml.safe_load(f)
    cfg = from_dict({"model": body})
    assert cfg.model.name == body["name"]
    for k in body:
        if k not in ("name", "cutoff", "n_features", "n_interactions", "n_rbf"):
            assert k in cfg.model.extra, k
    model = prepare_model(cfg)
    assert sum(p.numel() for p in model.parameters()) > 0


def test_run_config_composes_groups():
    cfg = from_yaml(os.path.join(ROOT, "train.yaml"))
    assert cfg.model.name == "schnet" and cfg.data.batch_size == 5 and cfg.optim.force_weight == 10.0
    cfg = from_yaml(os.path.join(ROOT, "train.yaml"), {"model.cutoff": 4.0})
    assert cfg.model.cutoff == 4.0
