"""MatGL TensorNet potentials (MatPES and others) converted into :class:`TensorNet`.

A MatGL potential directory holds ``model.json`` (``kwargs``: the potential's options, with the
wrapped model's class and ``init_args``) and ``state.pt`` (the weights; the trunk under ``model.``,
the energy standardisation as ``data_mean`` / ``data_std``, the element references as
``element_refs.property_offset``). Their TensorNet is this package's with three options set:
the smooth spherical-Bessel radial basis (or Gaussians), a gated energy network and no self
pairs. Conversion:

* architecture from ``init_args``: ``units`` -> ``n_features``, ``nblocks`` -> ``n_interactions``,
  ``cutoff``, the radial basis (``rbf_type`` / ``use_smooth`` / ``max_n`` or ``num_rbf``), the
  activation (SiLU only), ``element_types`` -> species, ``data_std`` -> ``energy_scale``;
* weights: trunk layers by name (``model.`` prefix), the element embedding rows placed at their
  atomic numbers, the gated network's dense layers (MatGL's stacks interleave activations: its
  layer ``2 i`` is this package's layer ``i``), and the ``3 F`` outputs of the last scalar layer
  of the embedding and of every filter network reordered from per-feature ``(f, part)`` to
  per-part ``(part, f)``.

Not converted (an error names them): other radial bases, the ``SO(3)`` group, state features,
several targets, a repulsion term, intensive targets, a constant energy offset. Parity:
``src/xnn/gnn/models/tensornet_foundation.py:44-224`` of the reference.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Optional, Tuple, Union

import torch

from ..data.elements import SYMBOLS
from .tensornet import TensorNet

_SILU = ("swish", "silu")


def _read(path: Union[str, Path]):
    p = Path(path)
    if p.is_file():
        p = p.parent
    meta = json.loads((p / "model.json").read_text())
    kwargs = meta["kwargs"]
    model = kwargs["model"]
    if model.get("@class") != "TensorNet":
        raise NotImplementedError(f"{p} holds a {model.get('@class')}, not a TensorNet")
    state = torch.load(p / "state.pt", map_location="cpu", weights_only=True)
    if isinstance(state, dict) and isinstance(state.get("state_dict"), dict):
        state = state["state_dict"]
    return p, kwargs, model["init_args"], state


def _options(p: Path, kwargs: dict, a: dict, state: dict) -> Tuple[dict, int]:
    bad = []
    rbf = str(a.get("rbf_type", "Gaussian")).lower()
    if rbf == "sphericalbessel" and a.get("use_smooth", False):
        extra, n_rbf = {"radial_basis": "smooth_bessel"}, int(a["max_n"])
    elif rbf == "gaussian":
        n_rbf, span = int(a.get("num_rbf", 32)), float(a["cutoff"]) + 1.0
        width = a.get("width", 0.5)
        extra = {"radial_basis": "gaussian", "rbf_max": span,
                 "gamma": float(width) if width is not None else (n_rbf - 1) / span}
    else:
        bad.append(f"radial basis {a.get('rbf_type')}")
        extra, n_rbf = {}, 0
    group = str(a.get("equivariance_invariance_group", "O(3)"))
    if group != "O(3)":
        # MatGL's edge vectors point to the neighbour, this package's from it: only an O(3) model
        # is the same model under the mirror image
        bad.append(f"the {group} group")
    for key, what in (("include_state", "state features"), ("is_intensive", "an intensive target")):
        if a.get(key, key == "is_intensive"):
            bad.append(what)
    if int(a.get("ntargets", 1)) != 1:
        bad.append("several targets")
    if kwargs.get("calc_repuls", False):
        bad.append("a repulsion term")
    if str(a.get("activation_type", "swish")) not in _SILU:
        bad.append(f"activation {a.get('activation_type')}")
    if float(state.get("data_mean", torch.tensor(0.0))) != 0.0:
        bad.append("a constant energy offset")
    if bad:
        raise NotImplementedError(f"{p}: not converted: {', '.join(bad)}")
    species = [SYMBOLS.index(s) for s in a["element_types"]]
    extra.update(self_pairs=False, activation="silu", equivariance_group="O(3)", readout="gated",
                 n_elements=max(128, max(species) + 1), energy_scale=float(state.get("data_std", torch.tensor(1.0))),
                 species=species)
    refs = state.get("element_refs.property_offset")
    if refs is not None:
        extra["atomic_energies"] = [float(v) for v in refs.reshape(-1)[:len(species)]]
    return extra, n_rbf


def _per_part(t: torch.Tensor, units: int) -> torch.Tensor:
    """``3 F`` rows in MatGL's per-feature order ``(f, part)`` -> per part ``(part, f)``."""
    return t.reshape(units, 3, *t.shape[1:]).transpose(0, 1).reshape(t.shape)


def convert_directory(path: Union[str, Path], dtype: Optional[torch.dtype] = None):
    """``(model, config_dict)``: the :class:`TensorNet` of a MatGL directory and the config
    ``model`` section that rebuilds it."""
    p, kwargs, a, state = _read(path)
    extra, n_rbf = _options(p, kwargs, a, state)
    cfg = {"name": "tensornet", "cutoff": float(a["cutoff"]), "n_features": int(a["units"]),
           "n_interactions": int(a["nblocks"]), "n_rbf": n_rbf, "extra": extra}
    dtype = state["model.linear.weight"].dtype if dtype is None else dtype
    from ..config import from_dict
    previous = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        model = TensorNet.from_config(from_dict({"model": cfg}).model)
    finally:
        torch.set_default_dtype(previous)
    own = model.state_dict()
    new = {}
    for name in own:
        if name.startswith(("tensor_embedding.", "layers.", "out_norm.", "linear.")):
            key = "model." + name
            if name == "tensor_embedding.emb.weight":
                emb = own[name].clone()
                emb[torch.tensor(extra["species"])] = state[key].to(emb.dtype)
                new[name] = emb
            elif key in state:
                new[name] = state[key]
    for branch, theirs in (("mlp", "layers"), ("gate", "gates")):
        i = 0
        while f"readout.{branch}.layers.{i}.weight" in own:
            for q in ("weight", "bias"):
                new[f"readout.{branch}.layers.{i}.{q}"] = state[f"model.final_layer.gated.{theirs}.{2 * i}.{q}"]
            i += 1
    units = model.n_features
    for name in ["tensor_embedding.linears_scalar.1"] + [f"layers.{i}.linears_scalar.2" for i in range(int(a["nblocks"]))]:
        for q in ("weight", "bias"):
            new[f"{name}.{q}"] = _per_part(new[f"{name}.{q}"], units)
    kept = ("rbf.", "energy_", "atom_ref.", "cutoff_fn.")
    missing = [n for n in own if n not in new and not n.startswith(kept)]
    if missing:
        raise KeyError(f"{p}: no weights for {missing}")
    model.load_state_dict({**own, **{k: v.to(own[k].dtype) for k, v in new.items()}})
    return model, cfg
