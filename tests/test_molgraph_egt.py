"""Molecular graphs from explicit bonds and the EGT trunk against the reference implementation."""
import numpy as np
import pytest
import torch

from ref_oracle import load_same_weights, ref_module
from xnn_b200.featurizers.molgraph import molecular_graph_from_bonds


def _toluene():
    # ring C0..C5 (aromatic), methyl C6, ring H 7..11, methyl H 12..14
    z = [6] * 7 + [1] * 8
    bonds = [(i, (i + 1) % 6) for i in range(6)] + [(0, 6)] + [(i, 6 + i) for i in range(1, 6)] + [(6, 12), (6, 13), (6, 14)]
    orders = [1.5] * 6 + [1.0] * 9
    return z, bonds, orders


def test_molecular_graph_features():
    z, bonds, orders = _toluene()
    g = molecular_graph_from_bonds(z, bonds, orders)
    assert g.n_atoms == 15 and g.total_charge == 0
    assert list(g.min_ring[:7]) == [6] * 6 + [0] and list(g.ring_degree[:7]) == [2] * 6 + [0]
    assert int(g.bond_in_ring.sum()) == 6
    assert len(g.impropers) == 6            # the six aromatic carbons have three neighbours
    # symmetry: ortho carbons 1 and 5 share a class, meta 2 and 4 too, methyl hydrogens one class
    assert g.atom_class[1] == g.atom_class[5] and g.atom_class[2] == g.atom_class[4]
    assert g.atom_class[12] == g.atom_class[13] == g.atom_class[14] and g.atom_class[1] != g.atom_class[2]
    assert len(g.pairs12) == len(bonds) and len(g.angles) == sum(d * (d - 1) // 2 for d in g.degree)
    ei = g.edge_index()
    assert ei.shape == (2, 2 * len(bonds)) and (ei[:, 0::2] == ei[::-1, 1::2]).all()


@pytest.mark.parametrize("jk", ["cat", "last", None])
def test_egt_matches_reference(jk):
    ref_egt = ref_module("xnn.gnn.models.egt")
    from xnn_b200.models.egt import MolecularGraphTransformer
    z, bonds, orders = _toluene()
    g = molecular_graph_from_bonds(z, bonds, orders, formal_charges=[0] * 15)
    kw = dict(atom_dim=8, feature_dim=4, node_mlp=(16, 24, 2), edge_mlp=(16, 12, 2), hidden=24, layers=2, heads=3,
              head_dim=4, ffn=(16, 2), out_dim=24 if jk is None else 10, jumping_knowledge=jk)
    torch.manual_seed(0)
    ref = ref_egt.MolecularGraphTransformer(**kw).double()
    mine = MolecularGraphTransformer(**kw).double()
    load_same_weights(mine, ref)
    args = (torch.as_tensor(g.node_features()), torch.as_tensor(g.edge_features()), torch.as_tensor(g.edge_index()),
            torch.as_tensor(g.atom_class), torch.as_tensor(g.edge_class))
    (x, e), (xr, er) = mine(*args), ref(*args)
    torch.testing.assert_close(x, xr, rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(e, er, rtol=1e-10, atol=1e-12)
