"""NequIP: symmetry, forces, and the config-1 training path (CPU)."""
import torch

from xnn_b200.config import from_dict
from xnn_b200.data import AtomicDataset, collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput, build_model
from xnn_b200.models.nequip import NequIP


def _model():
    return NequIP(species=[1, 6, 8], cutoff=5.0, l_max=2, n_layers=3, num_features=8, n_rbf=8,
                  avg_num_neighbors=10.0)


def test_nequip_equivariance_and_forces():
    torch.set_default_dtype(torch.float64)
    try:
        m = _model()
        f = ForceStressOutput(m)
        g = collate([structure_to_graph(s, 5.0) for s in synthetic.small_organic(2, seed=3)])
        o = f(g.clone())
        q, _ = torch.linalg.qr(torch.randn(3, 3))
        q = q * torch.sign(torch.linalg.det(q))
        g2 = g.clone()
        g2.pos = g2.pos @ q.T
        o2 = f(g2)
        torch.testing.assert_close(o["energy"], o2["energy"], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(o["forces"] @ q.T, o2["forces"], rtol=1e-9, atol=1e-9)
        # parity: reflect through the origin
        g3 = g.clone()
        g3.pos = -g3.pos
        torch.testing.assert_close(o["energy"], f(g3)["energy"], rtol=1e-10, atol=1e-10)
        # finite differences
        h = 1e-5
        gp, gm = g.clone(), g.clone()
        gp.pos[2, 1] += h
        gm.pos[2, 1] -= h
        fd = -(m(gp)["energy"].sum() - m(gm)["energy"].sum()).detach() / (2 * h)
        assert abs(float(fd) - float(o["forces"][2, 1])) < 1e-6
    finally:
        torch.set_default_dtype(torch.float32)


def test_nequip_config1_trains(tmp_path):
    cfg = from_dict({"model": {"name": "nequip", "cutoff": 5.0, "n_features": 8, "n_interactions": 3, "n_rbf": 8,
                               "extra": {"species": [1, 6, 8], "l_max": 2, "avg_num_neighbors": 10.0}},
                     "optim": {"epochs": 2, "force_weight": 100.0, "lr": 5e-3},
                     "data": {"batch_size": 5}, "output_dir": str(tmp_path), "device": "cpu",
                     "trainer": {"loggers": []}})
    m = build_model(cfg)
    assert isinstance(m, NequIP)
    from xnn_b200.train import Trainer
    tr = Trainer(cfg, AtomicDataset(synthetic.small_organic(20, seed=1), 5.0))
    hist = tr.fit()
    assert (tmp_path / "best.pt").exists() and (tmp_path / "last.pt").exists()
    assert hist["train/loss"] > 0
