"""mace-torch conversion: an upstream-shaped module (mace-torch attribute names: weights_max and
descending lower orders, n pi / r_max Bessel weights, per-head readouts, scale_shift,
atomic_energies_fn) assembled around a MACE of this package converts back to the same energies
and forces; multi-head slicing picks one head's rows."""
import math
import types

import pytest
import torch
from torch import nn
from torch.nn import functional as F

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.mace import MACE
from xnn_b200.models.mace_foundation import from_mace_torch, model_config_dict


def _named(name, **attrs):
    cls = type(name, (nn.Module,), {})
    m = cls()
    for k, v in attrs.items():
        if isinstance(v, torch.Tensor):
            m.register_buffer(k, v)
        else:
            setattr(m, k, v)
    return m


def _upstream(m: MACE, species):
    up = _named("ScaleShiftMACE")
    up.register_buffer("atomic_numbers", torch.tensor(species))
    up.r_max = m.edge_feat.cutoff
    up.num_interactions = len(m.interactions)
    rbf = m.edge_feat.rbf
    up.radial_embedding = _named("RadialEmbeddingBlock", apply_cutoff=True,
                                 bessel_fn=_named("BesselBasis", bessel_weights=rbf.freqs / rbf.cutoff,
                                                  prefactor=rbf.norm),
                                 cutoff_fn=_named("PolynomialCutoff", p=float(m.edge_feat.envelope.p)),
                                 distance_transform=None)
    up.interactions = m.interactions
    for blk in up.interactions:
        blk.conv_tp_weights.hs = list(blk.conv_tp_weights.hs)
    prods = []
    for pr in m.products:
        cons = []
        for c in pr.symmetric_contractions.contractions:
            k = c.correlation
            uc = _named("Contraction", correlation=k)
            uc.weights_max = nn.Parameter(c.weights[k - 1].detach().clone())
            uc.weights = nn.ParameterList([nn.Parameter(c.weights[nu - 1].detach().clone()) for nu in range(k - 1, 0, -1)])
            for nu in range(1, k + 1):
                uc.register_buffer(f"U_matrix_{nu}", c.U(nu).clone())
            cons.append(uc)
        sc = _named("SymmetricContraction")
        sc.contractions = nn.ModuleList(cons)
        prods.append(_named("EquivariantProductBasisBlock", symmetric_contractions=sc, linear=pr.linear))
    up.products = nn.ModuleList(prods)
    last = m.readouts[-1]
    last.hidden_irreps = str(last.linear_1.irreps_out)
    last.non_linearity.acts = [F.silu]
    up.readouts = m.readouts
    up.scale_shift = _named("ScaleShiftBlock", scale=torch.tensor(m.scale_shift.scale.item()),
                            shift=torch.tensor(m.scale_shift.shift.item()))
    zs = torch.tensor(species)
    up.atomic_energies_fn = _named("AtomicEnergiesBlock",
                                   atomic_energies=m.atom_ref.weight.detach()[zs, 0].clone())
    up.node_embedding = _named("LinearNodeEmbeddingBlock", linear=m.node_embedding)
    return up


def _eval(model):
    mols = synthetic.organic_molecules(2, seed=8, n_min=6, n_max=14)
    b = collate([structure_to_graph(s, 4.5) for s in mols])
    out = ForceStressOutput(model).eval()(b)
    return out["energy"].detach(), out["forces"].detach()


def test_round_trip_through_upstream_layout():
    torch.set_default_dtype(torch.float64)
    try:
        species = [1, 6, 7, 8, 9, 16, 17]
        torch.manual_seed(0)
        m = MACE(species=species, cutoff=4.5, num_channels=16, max_ell=2, correlation=3, n_rbf=8,
                 avg_num_neighbors=7.0, atomic_energies=[-13.6, -1029.0, -1484.0, -2041.0, -2700.0, -10800.0, -12500.0],
                 scale=1.3, shift=0.2)
        with torch.no_grad():
            for p in m.parameters():
                p.add_(0.05 * torch.randn_like(p))
        e0, f0 = _eval(m)
        conv = from_mace_torch(_upstream(m, species))
        e1, f1 = _eval(conv)
        torch.testing.assert_close(e1, e0, rtol=1e-12, atol=1e-9)
        torch.testing.assert_close(f1, f0, rtol=1e-10, atol=1e-11)
        cfg = model_config_dict(conv)
        assert cfg["name"] == "mace" and cfg["extra"]["correlation"] == [3, 3]
    finally:
        torch.set_default_dtype(torch.float32)


def test_multi_head_slice():
    torch.set_default_dtype(torch.float64)
    try:
        species = [1, 6, 7, 8, 9, 16, 17]
        torch.manual_seed(1)
        m = MACE(species=species, cutoff=4.0, num_channels=8, max_ell=1, correlation=2, MLP_irreps="16x0e")
        ref_w2 = m.readouts[-1].linear_2.weight.detach().clone()
        ref_w0 = m.readouts[0].linear.weight.detach().clone()
        up = _upstream(m, species)          # shares m's modules: m is altered below
        up.heads = ["a", "b"]
        with pytest.raises(ValueError, match="heads"):
            from_mace_torch(up)
        # two heads: every readout doubled along its output; the MLP split in two halves
        for ro in up.readouts[:-1]:
            w = ro.linear.weight.detach().reshape(-1, 1)
            ro.linear.weight = nn.Parameter(torch.cat([w, 2.0 * w], 1).reshape(-1))
        last = up.readouts[-1]
        w1 = last.linear_1.weight.detach().reshape(-1, 16)
        last.linear_1.weight = nn.Parameter(torch.cat([w1, w1], 1).reshape(-1))
        last.hidden_irreps = "32x0e"
        w2 = last.linear_2.weight.detach().reshape(16, 1)
        W2 = torch.zeros(32, 2, dtype=w2.dtype)
        W2[:16, 0:1] = w2 * math.sqrt(2.0)
        W2[16:, 1:2] = 3.0 * w2 * math.sqrt(2.0)
        last.linear_2.weight = nn.Parameter(W2.reshape(-1))
        up.atomic_energies_fn.atomic_energies = torch.stack([up.atomic_energies_fn.atomic_energies] * 2)
        a = from_mace_torch(up, head="a")
        b = from_mace_torch(up, head="b")
        torch.testing.assert_close(a.readouts[-1].linear_2.weight.detach(), ref_w2)
        torch.testing.assert_close(b.readouts[-1].linear_2.weight.detach(), 3.0 * ref_w2)
        torch.testing.assert_close(b.readouts[0].linear.weight.detach(), 2.0 * ref_w0)
    finally:
        torch.set_default_dtype(torch.float32)
