"""Model hub: portable checkpoints, a registry of named models, downloads, ``from_pretrained``.

A source is a local checkpoint path, a registered name (entries of ``$XNN_B200_HUB``, a directory
of portable model directories, one per name, or names given to :func:`register_pretrained`), or a
URL / Zenodo DOI, downloaded once into the model cache (:mod:`xnn_b200.hub.fetch`).
"""
from __future__ import annotations

import os
from pathlib import Path
from typing import Dict, Optional, Union

from torch import nn

from .card import CARD_FILE, CONFIG_FILE, WEIGHTS_FILE, ModelCard
from .checkpoint import (Checkpoint, build_potential, config_to_dict, load_checkpoint, read_config,
                         save_pretrained, write_config)
from .fetch import fetch_model, is_remote, model_cache_dir

_REGISTRY: Dict[str, Path] = {}


def register_pretrained(name: str, path: Union[str, Path]) -> None:
    """Name a local model directory / checkpoint, or a URL / DOI fetched on first use."""
    _REGISTRY[name] = path if is_remote(path) else Path(path)


def list_pretrained() -> Dict[str, Path]:
    out = dict(_REGISTRY)
    root = os.environ.get("XNN_B200_HUB")
    if root and os.path.isdir(root):
        for d in sorted(Path(root).iterdir()):
            if (d / CARD_FILE).exists() or (d / WEIGHTS_FILE).exists():
                out.setdefault(d.name, d)
    return out


def resolve(source: Union[str, Path], cache_dir: Optional[Union[str, Path]] = None) -> Path:
    if is_remote(source):
        return fetch_model(source, cache_dir=cache_dir)
    p = Path(source).expanduser()
    if p.exists():
        return p
    known = list_pretrained()
    if str(source) in known:
        v = known[str(source)]
        return fetch_model(str(v), cache_dir=cache_dir) if is_remote(v) else Path(v)
    raise FileNotFoundError(f"{source!r} is neither a checkpoint path, a URL / DOI nor a registered model "
                            f"(known: {sorted(known)})")


def from_pretrained(source: Union[str, Path], wrap: bool = True, dtype=None,
                    cache_dir: Optional[Union[str, Path]] = None) -> nn.Module:
    """The model of a checkpoint path, registered name, URL or Zenodo DOI; ``wrap`` keeps the
    force/stress wrapper."""
    ck = load_checkpoint(resolve(source, cache_dir=cache_dir))
    if ck.config is None:
        raise ValueError(f"{source}: a bare state dict carries no config; use build_potential(config, sd)")
    pot = build_potential(ck.config, ck.state_dict, dtype=dtype)
    return pot if wrap else pot.model


__all__ = ["Checkpoint", "ModelCard", "build_potential", "config_to_dict", "fetch_model", "from_pretrained",
           "is_remote", "list_pretrained", "model_cache_dir",
           "load_checkpoint", "read_config", "register_pretrained", "resolve", "save_pretrained", "write_config",
           "CARD_FILE", "CONFIG_FILE", "WEIGHTS_FILE"]
