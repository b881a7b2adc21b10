"""Reading, writing and rebuilding models from checkpoints.

Formats follow the reference's ``src/xnn/common/models/hub/checkpoint.py`` (``load_checkpoint``
at ``:239``, ``save_pretrained`` at ``:305``, ``build_potential`` at ``:435``) so checkpoints
move between the two:

* a portable model directory: ``card.json``, ``config.yaml`` (plain YAML of the run config) and
  ``model.pt`` (a state dict, loadable with ``torch.load(weights_only=True)``);
* a trainer checkpoint ``{"model": state_dict, "cfg": dict}`` (``best.pt`` / ``last.pt``);
* a bare state dict.

State dicts are in the :class:`~xnn_b200.models.ForceStressOutput` layout (keys ``model.*``).
"""
from __future__ import annotations

import dataclasses
import hashlib
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, Optional, Union

import torch
import yaml
from torch import nn

from .card import CARD_FILE, CONFIG_FILE, WEIGHTS_FILE, ModelCard


@dataclass
class Checkpoint:
    config: Any
    state_dict: Dict[str, torch.Tensor]
    card: Optional[ModelCard]
    path: Path


def config_to_dict(config: Any) -> Dict[str, Any]:
    """A plain-data dict of a :class:`~xnn_b200.config.Config` (or a dict)."""
    if config is None:
        return {}
    if isinstance(config, dict):
        return dict(config)
    if hasattr(config, "to_dict"):
        return config.to_dict()
    if dataclasses.is_dataclass(config):
        return dataclasses.asdict(config)
    raise TypeError(f"cannot serialise a config of type {type(config).__name__}")


def write_config(config: Any, path: Union[str, Path]) -> Path:
    p = Path(path)
    p.write_text(yaml.safe_dump(config_to_dict(config), sort_keys=False))
    return p


def read_config(path: Union[str, Path]):
    from ..config import from_dict
    with open(path) as f:
        return from_dict(yaml.safe_load(f) or {})


def _md5(path: Path) -> str:
    h = hashlib.md5()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _as_config(cfg):
    if cfg is None or not isinstance(cfg, dict):
        return cfg
    from ..config import from_dict
    return from_dict(cfg)


def load_checkpoint(path: Union[str, Path]) -> Checkpoint:
    """Read a portable directory, a trainer checkpoint or a bare state dict."""
    p = Path(path)
    if p.is_dir():
        card = ModelCard.read(p / CARD_FILE) if (p / CARD_FILE).exists() else None
        cfg = read_config(p / CONFIG_FILE) if (p / CONFIG_FILE).exists() else None
        state = torch.load(p / WEIGHTS_FILE, map_location="cpu", weights_only=True)
        # the directory's weights file holds {"model": state_dict}; older or hand-written
        # directories may hold the bare state dict
        sd = state["model"] if isinstance(state, dict) and isinstance(state.get("model"), dict) else state
        return Checkpoint(cfg, sd, card, p)
    obj = torch.load(p, map_location="cpu", weights_only=False)
    if isinstance(obj, dict) and "model" in obj and isinstance(obj["model"], dict):
        return Checkpoint(_as_config(obj.get("cfg")), obj["model"], None, p)
    if isinstance(obj, dict) and all(isinstance(v, torch.Tensor) for v in obj.values()):
        return Checkpoint(None, obj, None, p)
    raise ValueError(f"{p} is not a model checkpoint")


def wrapped_state_dict(model: nn.Module) -> Dict[str, torch.Tensor]:
    """State dict in the ``ForceStressOutput`` layout (``model.*`` keys)."""
    from ..models.outputs import ForceStressOutput
    sd = model.state_dict()
    if isinstance(model, ForceStressOutput):
        return {k: v.detach().cpu() for k, v in sd.items()}
    return {f"model.{k}": v.detach().cpu() for k, v in sd.items()}


def save_pretrained(model: Union[nn.Module, str, Path], path: Union[str, Path], config: Any = None,
                    card: Optional[ModelCard] = None) -> Path:
    """Write a portable model directory from a model (with its ``config``) or a checkpoint file."""
    out = Path(path)
    out.mkdir(parents=True, exist_ok=True)
    if isinstance(model, (str, Path)):
        ck = load_checkpoint(model)
        sd, config = ck.state_dict, config if config is not None else ck.config
        card = card or ck.card
    else:
        sd = wrapped_state_dict(model)
    if config is None:
        raise ValueError("save_pretrained needs the model's config to rebuild it")
    torch.save({"model": dict(sd)}, out / WEIGHTS_FILE)
    write_config(config, out / CONFIG_FILE)
    cfg = _as_config(config_to_dict(config))
    card = card or ModelCard()
    card.model = card.model or cfg.model.name
    card.cutoff = card.cutoff if card.cutoff is not None else float(cfg.model.cutoff)
    card.species = card.species or list((cfg.model.extra or {}).get("species", []))
    card.md5 = _md5(out / WEIGHTS_FILE)
    card.write(out / CARD_FILE)
    return out


def build_potential(config: Any, state_dict: Dict[str, torch.Tensor], dtype: Optional[torch.dtype] = None,
                    compute_stress: bool = True) -> nn.Module:
    """The model of ``config`` with the weights of ``state_dict``, wrapped for forces/stress."""
    from ..models.outputs import ForceStressOutput
    from ..models.registry import prepare_model
    cfg = _as_config(config_to_dict(config))
    extra = dict(cfg.model.extra or {})
    extra.pop("pretrained", None)
    cfg.model.extra = extra
    model = prepare_model(cfg)
    wrapped = ForceStressOutput(model, compute_stress=compute_stress)
    missing, unexpected = wrapped.load_state_dict(state_dict, strict=False)
    real_missing = [k for k in missing if not k.endswith("_fast_consts")]
    if real_missing or unexpected:
        raise RuntimeError(f"checkpoint does not match the model: missing {real_missing[:5]}, "
                           f"unexpected {list(unexpected)[:5]}")
    if dtype is not None:
        wrapped = wrapped.to(dtype)
    return wrapped.eval()
