"""ByteFF-Pol against the reference: the same weights and molecular graphs give the same predicted
parameters, energy terms (repulsion, dispersion, electrostatics, charge transfer, polarization),
induced dipoles and forces; plus the dipoles' stationarity and an ensemble."""
import pytest
import torch

from ref_oracle import load_same_weights, ref_graph, ref_module
from test_byteff import BONDS, ORDERS, SMALL, Z, _batch, _graphs
from xnn_b200.ffnn.byteff_pol import ByteFFPol
from xnn_b200.models import ForceStressOutput

POL_SMALL = dict(graph=SMALL["graph"], bonded=dict(pre=(24, 24, 2), out=(16, 2)),
                 nonbonded=dict(pre=(24, 24, 2), out=(16, 2)))


@pytest.fixture(autouse=True)
def _f64():
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(prev)


@pytest.mark.parametrize("members", [1, 2])
def test_byteff_pol_matches_reference(members):
    rb = ref_module("xnn.hybnn.models.byteff")
    torch.manual_seed(0)
    ref = rb.ByteFFPol(use_fast=False, members=members, **POL_SMALL).double()
    mine = ByteFFPol(members=members, **POL_SMALL).double().bind(Z, BONDS, ORDERS)
    load_same_weights(mine, ref)
    graphs = _graphs()
    species = [(0, list(range(7))), (1, [7, 8, 9]), (1, [10, 11, 12])]
    ref._bind_graphs(graphs, species)
    ref._bind_hypervalent(graphs, species, None)
    b = _batch()
    outs = ref_module("xnn.common.models.outputs")
    ref.eval(), mine.eval()
    o_ref = outs.ForceStressOutput(ref)(ref_graph(b))
    o = ForceStressOutput(mine)(b.clone())
    for k in ("energy", "forces", "charges", "induced_dipoles", "e_bond", "e_angle", "e_torsion", "e_improper",
              "e_repulsion", "e_dispersion", "e_electrostatics", "e_charge_transfer", "e_polarization"):
        torch.testing.assert_close(o[k].double(), o_ref[k].double(), rtol=1e-9, atol=1e-10, msg=k)
    assert float(o["e_polarization"].abs().sum()) > 0 and float(o["e_charge_transfer"].abs().sum()) > 0
    pm, pr = mine.predicted_parameters(), ref.predicted_parameters()
    for k in pm:
        torch.testing.assert_close(pm[k], pr[k], rtol=1e-9, atol=1e-10, msg=k)


def test_forward_dipoles_and_energy_sign():
    """The forward pass reports the solve's dipoles; the induction energy -k/2 mu.E is negative."""
    torch.manual_seed(1)
    m = ByteFFPol(**POL_SMALL).double().bind(Z, BONDS, ORDERS).eval()
    b = _batch(n=1)
    with torch.no_grad():
        P = {k: m.predicted_parameters()[k][m._atom_src] for k in ("charge", "alpha", "damp")}
        mu, field = m._dipoles(b.pos.view(1, -1, 3), P["charge"][None], P["alpha"][None], P["damp"][None])
        out = m(b)
    assert torch.allclose(out["induced_dipoles"], mu.reshape(-1, 3), atol=1e-12)
    assert float(out["e_polarization"].sum()) < 0.0
    assert abs(float(out["charges"].sum())) < 1e-10                # neutral molecules
