"""MatGL TensorNet directories: a directory written in MatGL's layout (model.json + state.pt,
per-feature 3F rows, interleaved gated stacks, embedding rows per element type) from a model of
this package converts back to the same energies and forces; unsupported options are refused."""
import json

import pytest
import torch

from xnn_b200.data import collate, structure_to_graph, synthetic
from xnn_b200.data.elements import SYMBOLS
from xnn_b200.models import ForceStressOutput
from xnn_b200.models.tensornet import TensorNet
from xnn_b200.models.tensornet_foundation import convert_directory


def _write_matgl(model: TensorNet, species, path, **overrides):
    units = model.n_features
    own = model.state_dict()
    state = {}
    for name, t in own.items():
        if name.startswith(("tensor_embedding.", "layers.", "out_norm.", "linear.")):
            v = t.clone()
            if name == "tensor_embedding.emb.weight":
                v = v[torch.tensor(species)]
            if any(name.startswith(p) for p in ["tensor_embedding.linears_scalar.1."] +
                   [f"layers.{i}.linears_scalar.2." for i in range(len(model.layers))]):
                v = v.reshape(3, units, *v.shape[1:]).transpose(0, 1).reshape(v.shape)   # per part -> per feature
            state["model." + name] = v
    for branch, theirs in (("mlp", "layers"), ("gate", "gates")):
        i = 0
        while f"readout.{branch}.layers.{i}.weight" in own:
            for q in ("weight", "bias"):
                state[f"model.final_layer.gated.{theirs}.{2 * i}.{q}"] = own[f"readout.{branch}.layers.{i}.{q}"].clone()
            i += 1
    state["data_mean"] = torch.tensor(0.0)
    state["data_std"] = model.energy_scale.clone()
    state["element_refs.property_offset"] = model.atom_ref.weight.detach()[torch.tensor(species), 0].clone()
    args = {"units": units, "nblocks": len(model.layers), "cutoff": model.cutoff, "rbf_type": "SphericalBessel",
            "use_smooth": True, "max_n": model.rbf.n_rbf if hasattr(model.rbf, "n_rbf") else 6,
            "activation_type": "swish", "equivariance_invariance_group": "O(3)", "is_intensive": False,
            "ntargets": 1, "element_types": [SYMBOLS[z] for z in species]}
    args.update(overrides)
    (path / "model.json").write_text(json.dumps({"kwargs": {"model": {"@class": "TensorNet", "init_args": args},
                                                            "calc_repuls": False}}))
    torch.save(state, path / "state.pt")


def _eval(model):
    s = synthetic.triclinic_crystals(2, seed=4, n_min=8, n_max=16, z_max=20, labels=False)
    b = collate([structure_to_graph(x, 5.0) for x in s])
    out = ForceStressOutput(model).eval()(b)
    return out["energy"].detach(), out["forces"].detach()


def test_round_trip(tmp_path):
    torch.set_default_dtype(torch.float64)
    try:
        species = list(range(1, 21))
        torch.manual_seed(0)
        m = TensorNet(n_features=8, n_interactions=2, n_rbf=6, cutoff=5.0, radial_basis="smooth_bessel",
                      readout="gated", self_pairs=False, species=species, n_elements=128,
                      atomic_energies=[0.1 * z for z in species], energy_scale=1.7)
        with torch.no_grad():
            for p in m.parameters():
                p.add_(0.05 * torch.randn_like(p))
            emb = m.tensor_embedding.emb.weight
            keep = emb[torch.tensor(species)].clone()
            emb.zero_()
            emb[torch.tensor(species)] = keep
            m.atom_ref.weight.zero_()
            m.atom_ref.weight[torch.tensor(species), 0] = torch.tensor([0.1 * z for z in species])
        _write_matgl(m, species, tmp_path)
        conv, cfg = convert_directory(tmp_path)
        assert cfg["extra"]["radial_basis"] == "smooth_bessel" and cfg["extra"]["self_pairs"] is False
        e0, f0 = _eval(m)
        e1, f1 = _eval(conv)
        torch.testing.assert_close(e1, e0, rtol=1e-12, atol=1e-10)
        torch.testing.assert_close(f1, f0, rtol=1e-10, atol=1e-11)
    finally:
        torch.set_default_dtype(torch.float32)


def test_refused_options(tmp_path):
    m = TensorNet(n_features=8, n_interactions=1, n_rbf=6, cutoff=5.0, radial_basis="smooth_bessel",
                  readout="gated", self_pairs=False, species=[1, 8], n_elements=128)
    _write_matgl(m, [1, 8], tmp_path, equivariance_invariance_group="SO(3)", is_intensive=True)
    with pytest.raises(NotImplementedError, match="SO\\(3\\).*intensive|intensive.*SO\\(3\\)"):
        convert_directory(tmp_path)
