"""TensorNet: symmetry, forces, periodic stress and the config-3 training path (CPU)."""
import torch

from xnn_b200.config import from_dict
from xnn_b200.data import AtomicDataset, collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.tensornet import TensorNet


def test_tensornet_symmetry_forces_stress():
    torch.set_default_dtype(torch.float64)
    try:
        m = TensorNet(n_features=8, n_interactions=2, n_rbf=8, cutoff=5.0, n_elements=90)
        f = ForceStressOutput(m, compute_stress=True)
        crys = synthetic.triclinic_crystals(2, seed=4, n_min=8, n_max=14, labels=False)
        g = collate([structure_to_graph(s, 5.0) for s in crys])
        o = f(g.clone())
        q, _ = torch.linalg.qr(torch.randn(3, 3))
        g2 = g.clone()
        g2.pos = g2.pos @ q.T
        g2.cell = g2.cell @ q.T
        o2 = f(g2)
        torch.testing.assert_close(o["energy"], o2["energy"], rtol=1e-9, atol=1e-9)
        torch.testing.assert_close(o["forces"] @ q.T, o2["forces"], rtol=1e-8, atol=1e-8)
        torch.testing.assert_close(q @ o["stress"] @ q.T, o2["stress"], rtol=1e-8, atol=1e-9)
        h = 1e-5
        gp, gm = g.clone(), g.clone()
        gp.pos[1, 0] += h
        gm.pos[1, 0] -= h
        fd = -(m(gp)["energy"].sum() - m(gm)["energy"].sum()).detach() / (2 * h)
        assert abs(float(fd) - float(o["forces"][1, 0])) < 1e-6
    finally:
        torch.set_default_dtype(torch.float32)


def test_tensornet_config3_trains_with_stress(tmp_path):
    cfg = from_dict({"model": {"name": "tensornet", "cutoff": 5.0, "n_features": 16, "n_interactions": 2,
                               "n_rbf": 16, "extra": {"n_elements": 90}},
                     "optim": {"epochs": 1, "stress_weight": 1.0, "lr": 1e-3},
                     "data": {"batch_size": 4}, "output_dir": str(tmp_path), "device": "cpu",
                     "trainer": {"loggers": []}})
    from xnn_b200.train import Trainer
    ds = AtomicDataset(synthetic.triclinic_crystals(10, seed=2, n_min=8, n_max=20), 5.0)
    tr = Trainer(cfg, ds)
    assert tr.module.compute_stress
    tr.fit()
    assert (tmp_path / "last.pt").exists()
