"""ByteFF against the reference: the same weights and the same molecular graphs give the same
predicted parameters, energies, energy terms and forces (all pairs and with a cutoff, harmonic and
two-well bonded forms, ensembles); plus binding from bond lists and charge conservation."""
import numpy as np
import pytest
import torch

from ref_oracle import load_same_weights, ref_graph, ref_module
from xnn_b200.data import collate, structure_to_graph
from xnn_b200.ffnn.byteff import ByteFF, split_molecules
from xnn_b200.models import ForceStressOutput

SMALL = dict(graph=dict(atom_dim=8, feature_dim=4, node_mlp=(16, 24, 2), edge_mlp=(16, 12, 2), hidden=24, layers=2,
                        heads=4, head_dim=6, ffn=(24, 2), out_dim=20),
             bonded=dict(pre=(24, 24, 2), out=(16, 2)), nonbonded=dict(pre=(24, 24, 2), out=(16, 2)))

# acetaldehyde (carbonyl C: an improper), then two waters
Z = [6, 6, 8, 1, 1, 1, 1, 8, 1, 1, 8, 1, 1]
BONDS = [(0, 1), (1, 2), (0, 3), (0, 4), (0, 5), (1, 6), (7, 8), (7, 9), (10, 11), (10, 12)]
ORDERS = [1.0, 2.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0]
POS = np.array([[0.0, 0.0, 0.0], [1.50, 0.0, 0.0], [2.1, 1.05, 0.0], [-0.36, 1.0, 0.1], [-0.36, -0.5, 0.87],
                [-0.36, -0.5, -0.87], [2.05, -0.95, 0.0], [4.0, 0.5, 0.3], [4.96, 0.5, 0.3], [3.76, 1.43, 0.3],
                [0.5, 3.5, 1.0], [1.46, 3.5, 1.0], [0.26, 4.43, 1.0]])


def _batch(n=2, cutoff=6.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    structs = [{"pos": torch.tensor(POS) + 0.05 * torch.randn(len(Z), 3, generator=g, dtype=torch.float64),
                "atomic_numbers": torch.tensor(Z)} for _ in range(n)]
    return collate([structure_to_graph(s, cutoff) for s in structs])


def test_split_and_bind():
    assert split_molecules(len(Z), BONDS) == [list(range(7)), [7, 8, 9], [10, 11, 12]]
    torch.manual_seed(0)
    m = ByteFF(**SMALL).double().bind(Z, BONDS, ORDERS)
    assert m._u_features.shape[0] == 10              # the second water shares the first one's graph
    with torch.no_grad():
        q = m.predicted_parameters()["charge"][m._atom_src]
    for atoms in split_molecules(len(Z), BONDS):
        assert abs(float(q[atoms].sum())) < 1e-12      # neutral molecules stay neutral


@pytest.mark.parametrize("kw", [dict(), dict(bonded=dict(form="two_well"), members=2),
                                dict(cutoff=4.0, switch_width=1.0)])
def test_byteff_matches_reference(kw):
    rb = ref_module("xnn.hybnn.models.byteff")
    cfg = {**SMALL, **kw}
    if "bonded" in kw:
        cfg["bonded"] = {**SMALL["bonded"], **kw["bonded"]}
    torch.manual_seed(0)
    ref = rb.ByteFF(use_fast=False, **cfg).double()
    mine = ByteFF(**cfg).double().bind(Z, BONDS, ORDERS)
    load_same_weights(mine, ref)
    ref_graphs = [mine_graph for mine_graph in _graphs()]
    species = [(0, list(range(7))), (1, [7, 8, 9]), (1, [10, 11, 12])]
    ref._bind_graphs(ref_graphs, species)
    ref._bind_hypervalent(ref_graphs, species, None)
    b = _batch(cutoff=4.0 if "cutoff" in kw else 6.0)
    outs = ref_module("xnn.common.models.outputs")
    ref.eval(), mine.eval()
    o_ref = outs.ForceStressOutput(ref)(ref_graph(b))
    o = ForceStressOutput(mine)(b.clone())
    for k in ("energy", "forces", "charges", "e_bond", "e_angle", "e_torsion", "e_improper", "e_vdw", "e_coulomb",
              "e_vdw14", "e_coulomb14"):
        torch.testing.assert_close(o[k].double(), o_ref[k].double(), rtol=1e-9, atol=1e-10, msg=k)
    assert float(o["e_improper"].abs().sum()) > 0 and float(o["e_torsion"].abs().sum()) > 0
    pm, pr = mine.predicted_parameters(), ref.predicted_parameters()
    for k in pm:
        torch.testing.assert_close(pm[k], pr[k], rtol=1e-9, atol=1e-10, msg=k)


def _graphs():
    from xnn_b200.featurizers.molgraph import molecular_graph_from_bonds
    return [molecular_graph_from_bonds(Z[:7], BONDS[:6], ORDERS[:6]),
            molecular_graph_from_bonds([8, 1, 1], [(0, 1), (0, 2)])]


def test_training_gradients_reach_the_graph_network():
    torch.manual_seed(0)
    m = ByteFF(**SMALL).double().bind(Z, BONDS, ORDERS).train()
    out = ForceStressOutput(m).train()(_batch())
    loss = out["energy"].pow(2).sum() + out["forces"].pow(2).sum()
    loss.backward()
    g = m.members[0].graph.embedding.element.weight.grad
    assert g is not None and float(g.abs().sum()) > 0
