"""Convert ``mace-torch`` models (the MACE-MP / MACE-OFF foundation checkpoints) into :class:`MACE`.

Foundation MACE checkpoints are pickled ``mace.modules.models.ScaleShiftMACE`` (or ``MACE``)
modules. Since this MACE keeps the upstream block layout and parameter names, a conversion
reads the architecture off the upstream module, builds the same model here and copies the
weights block by block:

* architecture: species (``atomic_numbers``), ``r_max``, interaction count and classes, the
  radial basis (Bessel / Gaussian, its size and the envelope power), the distance transform,
  hidden irreps, ``max_ell`` (``edge_attrs_irreps``), the radial MLP widths, the correlation of
  every product, the readout MLP irreps and gate, ``avg_num_neighbors``, pair repulsion,
  reference energies and the scale / shift;
* weights: node embedding, every interaction block's state, the symmetric contractions
  (upstream keeps the top order as ``weights_max`` and the lower orders descending; here all
  orders ascend in one list), the product linears, the readouts, the distance-transform and
  ZBL buffers, and the Bessel frequencies as stored (upstream stores ``n pi / r_max``).

Multi-head checkpoints are cut to one head (``head=``): its reference energies, scale / shift and
readout rows, with the final readout's fan-in renormalised by ``sqrt(1 / n_heads)`` (the e3nn
linear normalises by the fan-in it was built with). Reading a checkpoint file needs the
``mace-torch`` package (the pickle names its classes); the conversion itself and the converted
model do not. Parity: ``src/xnn/gnn/models/mace_foundation.py:305-497`` of the reference.
"""
from __future__ import annotations

import math
from pathlib import Path
from typing import Optional, Tuple, Union

import torch
from torch import nn

from ..o3 import Irreps
from .mace import GATES, INTERACTIONS, MACE


def load_mace_torch(path: Union[str, Path]) -> nn.Module:
    """Unpickle a ``mace-torch`` checkpoint (needs the ``mace-torch`` package installed)."""
    try:
        import mace  # noqa: F401  (its classes are named by the pickle)
    except ModuleNotFoundError as err:
        raise ImportError("reading a mace-torch checkpoint needs the mace-torch package "
                          "(pip install mace-torch); convert it where that is installed and save the "
                          "result with xnn_b200.hub.save_pretrained") from err
    return torch.load(Path(path).expanduser(), map_location="cpu", weights_only=False)


def _head(upstream: nn.Module, head: Optional[str]) -> Tuple[int, int]:
    heads = [str(h) for h in getattr(upstream, "heads", ["Default"])]
    if head is None:
        if len(heads) != 1:
            raise ValueError(f"the checkpoint has {len(heads)} heads {heads}: pass head=<name>")
        return 0, 1
    if str(head) not in heads:
        raise ValueError(f"no head {head!r} in {heads}")
    return heads.index(str(head)), len(heads)


def _gate(fn) -> str:
    raw = getattr(fn, "f", fn)
    name = getattr(raw, "__name__", "")
    for key, g in GATES.items():
        if g is not None and (g is raw or getattr(g, "__name__", None) == name):
            return key
    raise NotImplementedError(f"readout gate {raw!r} is not one of {sorted(k for k in GATES if k)}")


def _scalar_rows(linear: nn.Module, n_out: int) -> torch.Tensor:
    """An all-scalar e3nn linear's flat weight as ``(fan_in, n_out)``."""
    return linear.weight.detach().reshape(-1, n_out)


def _copy_buffers(dst: nn.Module, src: nn.Module) -> None:
    have = dict(src.named_buffers())
    with torch.no_grad():
        for name, buf in dst.named_buffers():
            if name in have and have[name].shape == buf.shape:
                buf.copy_(have[name].to(buf.dtype))


def from_mace_torch(upstream: nn.Module, head: Optional[str] = None, dtype=None) -> MACE:
    """The :class:`MACE` equivalent of an upstream ``mace-torch`` model (see module notes)."""
    hi, n_heads = _head(upstream, head)
    up_dtype = next(upstream.parameters()).dtype
    species = [int(z) for z in upstream.atomic_numbers]
    r_max = float(upstream.r_max)
    T = int(upstream.num_interactions)
    emb = upstream.radial_embedding
    if not getattr(emb, "apply_cutoff", True):
        raise NotImplementedError("radial embeddings without the envelope (apply_cutoff=False) are not built here")
    radial_type = {"BesselBasis": "bessel", "GaussianBasis": "gaussian"}.get(type(emb.bessel_fn).__name__)
    if radial_type is None:
        raise NotImplementedError(f"radial basis {type(emb.bessel_fn).__name__}")
    n_rbf = int(emb.bessel_fn.bessel_weights.numel()) if radial_type == "bessel" else int(
        getattr(emb.bessel_fn, "num_basis", emb.out_dim))
    transform = getattr(emb, "distance_transform", None)
    t_name = "None" if transform is None else {"AgnesiTransform": "Agnesi", "SoftTransform": "Soft"}.get(
        type(transform).__name__)
    if t_name is None:
        raise NotImplementedError(f"distance transform {type(transform).__name__}")
    names = [type(b).__name__ for b in upstream.interactions]
    for nm in names:
        if nm not in INTERACTIONS:
            raise NotImplementedError(f"interaction block {nm} is not built here")
    if T >= 2 and len(set(names[1:])) > 1:
        raise NotImplementedError(f"mixed interaction blocks after the first: {names}")
    first = upstream.interactions[0]
    hidden = str(Irreps(str(first.hidden_irreps)))
    max_ell = Irreps(str(first.edge_attrs_irreps)).lmax
    radial_mlp = [int(h) for h in first.conv_tp_weights.hs[1:-1]]
    correlation = [int(p.symmetric_contractions.contractions[0].correlation) for p in upstream.products]
    readouts = list(upstream.readouts)
    if len(readouts) != max(T, 1) or not hasattr(readouts[-1], "linear_1"):
        raise NotImplementedError("readouts other than one per interaction, the last non-linear")
    last = readouts[-1]
    mlp = Irreps(str(last.hidden_irreps))
    if len(mlp) != 1 or mlp[0].ir.l != 0 or mlp[0].mul % n_heads:
        raise NotImplementedError(f"readout MLP irreps {mlp}")
    mlp_mul = mlp[0].mul // n_heads
    scale = shift = None
    if hasattr(upstream, "scale_shift"):
        sc, sh = upstream.scale_shift.scale, upstream.scale_shift.shift
        scale = float(torch.atleast_1d(sc)[hi if sc.ndim else 0])
        shift = float(torch.atleast_1d(sh)[hi if sh.ndim else 0])
    e0 = torch.atleast_2d(upstream.atomic_energies_fn.atomic_energies.detach().cpu())[hi]
    avgs = {float(b.avg_num_neighbors) for b in upstream.interactions}
    if len(avgs) > 1:
        raise NotImplementedError(f"per-layer avg_num_neighbors {sorted(avgs)}")
    kw = dict(species=species, cutoff=r_max, max_ell=max_ell, num_channels=Irreps(hidden).count("0e"), n_rbf=n_rbf,
              num_interactions=T, correlation=correlation, MLP_irreps=f"{mlp_mul}x0e", radial_MLP=radial_mlp,
              interaction=names[-1], interaction_first=names[0], gate=_gate(last.non_linearity.acts[0]),
              avg_num_neighbors=avgs.pop(), hidden_irreps=hidden, num_cutoff_basis=int(float(emb.cutoff_fn.p)),
              radial_type=radial_type, distance_transform=t_name, pair_repulsion=hasattr(upstream, "pair_repulsion"),
              atomic_energies=[float(v) for v in e0],
              scale=1.0 if scale is None else scale, shift=0.0 if shift is None else shift)
    if radial_type == "bessel":
        kw["rbf_prefactor"] = float(emb.bessel_fn.prefactor)
    previous = torch.get_default_dtype()
    torch.set_default_dtype(up_dtype)
    try:
        model = MACE(**kw)
    finally:
        torch.set_default_dtype(previous)
    with torch.no_grad():
        model.node_embedding.load_state_dict(upstream.node_embedding.linear.state_dict())
        for t in range(T):
            state = {k: v for k, v in upstream.interactions[t].state_dict().items() if k != "avg_num_neighbors"}
            model.interactions[t].load_state_dict(state)
            for mine, theirs in zip(model.products[t].symmetric_contractions.contractions,
                                    upstream.products[t].symmetric_contractions.contractions):
                c = correlation[t]
                mine.weights[c - 1].copy_(theirs.weights_max)
                for nu in range(1, c):
                    mine.weights[nu - 1].copy_(theirs.weights[c - 1 - nu])
                _copy_buffers(mine, theirs)
            model.products[t].linear.load_state_dict(upstream.products[t].linear.state_dict())
        for t, ro in enumerate(readouts[:-1]):
            model.readouts[t].linear.weight.copy_(_scalar_rows(ro.linear, n_heads)[:, hi])
        model.readouts[-1].linear_1.weight.copy_(
            _scalar_rows(last.linear_1, mlp[0].mul)[:, hi * mlp_mul:(hi + 1) * mlp_mul].reshape(-1))
        model.readouts[-1].linear_2.weight.copy_(
            _scalar_rows(last.linear_2, n_heads)[hi * mlp_mul:(hi + 1) * mlp_mul, hi] * math.sqrt(1.0 / n_heads))
        if transform is not None:
            _copy_buffers(model.distance_transform, transform)
        if kw["pair_repulsion"]:
            _copy_buffers(model.pair_repulsion_fn, upstream.pair_repulsion_fn)
        if radial_type == "bessel":
            model.edge_feat.rbf.freqs.copy_(emb.bessel_fn.bessel_weights.detach().reshape(-1)
                                            .to(model.edge_feat.rbf.freqs.dtype) * r_max)
    if dtype is not None:
        model = model.to(getattr(torch, dtype) if isinstance(dtype, str) else dtype)
    model._init_options = dict(kw)
    return model


def convert_mace_torch_file(path: Union[str, Path], out_dir: Union[str, Path], head: Optional[str] = None,
                           dtype=None) -> Path:
    """Convert a ``mace-torch`` checkpoint file and write it as a portable model directory."""
    from ..config import from_dict
    from ..hub import save_pretrained
    model = from_mace_torch(load_mace_torch(path), head=head, dtype=dtype)
    cfg = from_dict({"model": model_config_dict(model)})
    return save_pretrained(model, out_dir, config=cfg)


def model_config_dict(model: MACE) -> dict:
    """The config ``model`` section that rebuilds a converted model through ``MACE.from_config``."""
    opts = dict(getattr(model, "_init_options", {}))
    if not opts:
        raise ValueError("the model carries no record of its constructor options (convert it with from_mace_torch)")
    core = {"name": "mace", "cutoff": opts.pop("cutoff"), "n_features": opts.pop("num_channels"),
            "n_interactions": opts.pop("num_interactions"), "n_rbf": opts.pop("n_rbf")}
    opts["num_polynomial_cutoff"] = opts.pop("num_cutoff_basis")
    return {**core, "extra": opts}
