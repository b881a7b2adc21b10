"""Model hub: portable checkpoints, local registry of named models, ``from_pretrained``.

This build has no network access, so named models resolve to local directories: entries of
``$XNN_B200_HUB`` (a directory of portable model directories, one per name) or names
registered with :func:`register_pretrained`.
"""
from __future__ import annotations

import os
from pathlib import Path
from typing import Dict, Optional, Union

from torch import nn

from .card import CARD_FILE, CONFIG_FILE, WEIGHTS_FILE, ModelCard
from .checkpoint import (Checkpoint, build_potential, config_to_dict, load_checkpoint, read_config,
                         save_pretrained, write_config)

_REGISTRY: Dict[str, Path] = {}


def register_pretrained(name: str, path: Union[str, Path]) -> None:
    _REGISTRY[name] = Path(path)


def list_pretrained() -> Dict[str, Path]:
    out = dict(_REGISTRY)
    root = os.environ.get("XNN_B200_HUB")
    if root and os.path.isdir(root):
        for d in sorted(Path(root).iterdir()):
            if (d / CARD_FILE).exists() or (d / WEIGHTS_FILE).exists():
                out.setdefault(d.name, d)
    return out


def resolve(source: Union[str, Path]) -> Path:
    p = Path(source)
    if p.exists():
        return p
    known = list_pretrained()
    if str(source) in known:
        return known[str(source)]
    raise FileNotFoundError(f"{source!r} is neither a checkpoint path nor a registered model "
                            f"(known: {sorted(known)}); downloads are not available in this build")


def from_pretrained(source: Union[str, Path], wrap: bool = True, dtype=None) -> nn.Module:
    """The model of a checkpoint path or registered name; ``wrap`` keeps the force/stress wrapper."""
    ck = load_checkpoint(resolve(source))
    if ck.config is None:
        raise ValueError(f"{source}: a bare state dict carries no config; use build_potential(config, sd)")
    pot = build_potential(ck.config, ck.state_dict, dtype=dtype)
    return pot if wrap else pot.model


__all__ = ["Checkpoint", "ModelCard", "build_potential", "config_to_dict", "from_pretrained", "list_pretrained",
           "load_checkpoint", "read_config", "register_pretrained", "resolve", "save_pretrained", "write_config",
           "CARD_FILE", "CONFIG_FILE", "WEIGHTS_FILE"]
