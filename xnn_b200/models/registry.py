"""Model registry: ``@register_model(name)``, ``build_model(cfg)`` and ``prepare_model(cfg)``.

``prepare_model`` applies the ``extra`` add-ons the reference supports
(``src/xnn/common/models/registry.py:23,74,123``): ``pretrained`` weights,
``lora`` adapters, ``heads`` (multi-head readouts), ``dispersion`` (D3/D4 wrapper) and
``long_range`` (latent Ewald wrapper).
"""
from __future__ import annotations

from typing import Callable, Dict, Type

from torch import nn

MODELS: Dict[str, Type[nn.Module]] = {}


def register_model(name: str) -> Callable:
    def deco(cls):
        key = name.lower()
        if key in MODELS and MODELS[key] is not cls:
            raise KeyError(f"model {name!r} is already registered")
        MODELS[key] = cls
        cls.registry_name = key
        return cls
    return deco


def _ensure_families() -> None:
    # importing the families registers their models
    from . import families  # noqa: F401


def list_models():
    _ensure_families()
    return sorted(MODELS)


def get_model_class(name: str):
    _ensure_families()
    key = name.lower()
    if key not in MODELS:
        raise KeyError(f"unknown model {name!r}; registered: {sorted(MODELS)}")
    return MODELS[key]


def build_model(cfg) -> nn.Module:
    """The bare model of ``cfg`` (a :class:`ModelConfig`, or a :class:`Config`)."""
    mcfg = getattr(cfg, "model", cfg)
    return get_model_class(mcfg.name).from_config(mcfg)


def prepare_model(cfg) -> nn.Module:
    """The model with every add-on of ``cfg.extra`` applied (see module notes)."""
    mcfg = getattr(cfg, "model", cfg)
    model = build_model(mcfg)
    extra = dict(mcfg.extra or {})
    if extra.get("heads"):
        from ..train.finetune import MultiHead
        model = MultiHead(model, list(extra["heads"]))
    if extra.get("pretrained"):
        from ..hub import load_checkpoint
        state = load_checkpoint(extra["pretrained"])["model"]
        state = {k[len("model."):] if k.startswith("model.") else k: v for k, v in state.items()}
        model.load_state_dict(state, strict=False)
    if extra.get("lora"):
        from ..train.finetune import inject_lora
        spec = extra["lora"] if isinstance(extra["lora"], dict) else {}
        inject_lora(model, **spec)
    if extra.get("long_range"):
        from .les import LatentEwald
        spec = extra["long_range"] if isinstance(extra["long_range"], dict) else {}
        model = LatentEwald(model, **spec)
    if extra.get("dispersion"):
        model = add_dispersion(model, extra["dispersion"])
    return model


def add_dispersion(model, spec):
    """Wrap ``model`` (or ``None``: pure dispersion) in a D3 / D4 correction.

    ``spec`` is ``{"name": "d3" | "d4", **options}``, a bare name, or ``True`` (D4 defaults), as
    the reference's ``add_dispersion`` (``src/xnn/common/models/registry.py:438``)."""
    if isinstance(spec, str):
        spec = {"name": spec}
    opts = dict(spec) if isinstance(spec, dict) else {}
    name = str(opts.pop("name", "d4")).lower()
    if name == "d3":
        from .d3 import D3_KEYS, D3Dispersion
        return D3Dispersion(model, **{k: v for k, v in opts.items() if k in D3_KEYS})
    if name == "d4":
        from .d4 import D4Dispersion
        return D4Dispersion(model, **opts)
    raise KeyError(f"unknown dispersion model {name!r} (use 'd3' or 'd4')")
