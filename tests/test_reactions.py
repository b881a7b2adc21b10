"""Reaction-energy sets and losses against the reference implementation."""
import torch

from ref_oracle import ref_module
from xnn_b200.data import synthetic


def _data():
    mols = synthetic.organic_molecules(4, seed=3, labels=False)
    structs = [dict(m, name=f"m{i}", subset=("A" if i < 2 else "B")) for i, m in enumerate(mols)]
    reactions = [{"species": ["m0", "m1"], "stoichiometry": [-1, 1], "reference": 2.5, "subset": "A"},
                 {"species": ["m2", "m3", "m2"], "stoichiometry": [1, -2, 0.5], "reference": -4.0, "subset": "B"},
                 {"species": ["m1", "m0"], "stoichiometry": [2, -1], "reference": 1.0, "weight": 3.0, "subset": "A"}]
    return {"structures": structs, "reactions": reactions}


def test_reaction_losses_match_reference():
    ref = ref_module("xnn.common.train.reactions")
    from xnn_b200.train.reactions import ReactionSet
    data = _data()
    for wtmad2 in (False, True):
        a, b = ReactionSet.from_gmtkn55(data, wtmad2=wtmad2), ref.ReactionSet.from_gmtkn55(data, wtmad2=wtmad2)
        e = torch.tensor([0.3, -1.2, 2.0, 0.7], dtype=torch.float64)
        torch.testing.assert_close(a.stoichiometry(), b.stoichiometry())
        for delta in (0.0, 0.05):
            torch.testing.assert_close(a.loss(e, delta), b.loss(e, delta))
        torch.testing.assert_close(a.errors(e), b.errors(e))
        sub_a, sub_b = a.subset([2, 0]), b.subset([2, 0])
        assert [s["name"] for s in sub_a.structures] == [s["name"] for s in sub_b.structures]
        torch.testing.assert_close(sub_a.stoichiometry(), sub_b.stoichiometry())
    assert sum(len(x) for x in ReactionSet.from_gmtkn55(data).batches(2)) == 3


def test_trainer_with_reaction_term(tmp_path):
    from xnn_b200.config import from_dict
    from xnn_b200.data import AtomicDataset
    from xnn_b200.train import Trainer
    from xnn_b200.train.reactions import ReactionSet
    cfg = from_dict({"model": {"name": "schnet", "cutoff": 4.0, "n_features": 8, "n_interactions": 1, "n_rbf": 6},
                     "optim": {"epochs": 2, "lr": 1e-3, "reaction_weight": 0.5, "reaction_batch_size": 2},
                     "data": {"batch_size": 4}, "output_dir": str(tmp_path), "device": "cpu",
                     "trainer": {"loggers": []}})
    ds = AtomicDataset(synthetic.organic_molecules(12, seed=4), 4.0)
    rs = ReactionSet.from_gmtkn55(_data())
    tr = Trainer(cfg, ds, reactions=rs, val_reactions=rs)
    metrics = tr.fit()
    assert "val/reaction_mae" in metrics and metrics["val/reaction_mae"] > 0
