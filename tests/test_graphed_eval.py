"""Captured evaluation: ordinary on the CPU; on a GPU the replay agrees with ordinary evaluations,
the replay / ordinary trial picks one, and inputs slower than max_ms are never captured."""
import pytest
import torch

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.deploy.graphed_eval import PROBES, GraphedEvaluation
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.schnet import SchNet


def _setup(device):
    torch.manual_seed(0)
    model = ForceStressOutput(SchNet(n_features=16, n_interactions=2, n_rbf=8, cutoff=4.0)).to(device).eval()
    mols = synthetic.small_organic(3, seed=2)
    g = collate([structure_to_graph(s, 4.0) for s in mols]).to(device)
    g.pos = g.pos.float()
    return model, g


def test_cpu_evaluations_are_ordinary():
    model, g = _setup("cpu")
    ev = GraphedEvaluation(model)
    out = ev(g)
    ref = model(g)
    torch.testing.assert_close(out["energy"], ref["energy"].detach())
    assert ev.captures == 0


@pytest.mark.gpu
def test_replay_matches_and_trial_decides():
    model, g = _setup("cuda")
    ev = GraphedEvaluation(model, trial=2, max_ms=1e6)
    ref = {k: v.detach() for k, v in model(g).items() if torch.is_tensor(v)}
    out1 = ev(g)                 # timed probe: ordinary
    out2 = ev(g)                 # capture + trial, then the chosen evaluation
    assert ev.captures == 1 and set(ev.trial_ms) == {"replay", "ordinary"}
    for out in (out1, out2):
        torch.testing.assert_close(out["energy"], ref["energy"], rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(out["forces"], ref["forces"], rtol=1e-4, atol=1e-5)
    ev.release()


@pytest.mark.gpu
def test_slow_inputs_stay_ordinary():
    model, g = _setup("cuda")
    ev = GraphedEvaluation(model, max_ms=0.0)
    for _ in range(PROBES + 2):
        ev(g)
    assert ev.captures == 0 and ev.capturable is False
