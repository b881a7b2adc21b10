"""Typed configuration (``src/xnn/common/config/schema.py:40-539``).

``Config{model, data, optim, trainer, device, seed, output_dir, subtracted_dispersion}`` with
the reference's field names and defaults (MACE defaults in ``model.extra``); the data
cutoff follows the model cutoff. Loaders: :func:`from_dict`, :func:`from_yaml`,
:func:`from_argparse` (``--config file.yaml --set a.b=c``), with dotted overrides and
upstream key spellings translated (MACE-CLI ``r_max``, ``num_channels``, ``E0s``; NequIP
``num_layers``).
"""
from __future__ import annotations

import ast
import copy
import os
import warnings
from dataclasses import asdict, dataclass, field, fields, is_dataclass
from typing import Any, Dict, List, Optional


def _default_mace_extra() -> Dict[str, Any]:
    return {"species": [1, 6, 8], "max_ell": 3, "max_L": 0, "correlation": 3,
            "num_polynomial_cutoff": 5, "MLP_irreps": "16x0e", "radial_MLP": [64, 64, 64],
            "gate": "silu", "avg_num_neighbors": 1.0}


@dataclass
class ModelConfig:
    name: str = "mace"
    cutoff: float = 4.0
    n_features: int = 32
    n_interactions: int = 2
    n_rbf: int = 8
    extra: Optional[Dict[str, Any]] = None

    def __post_init__(self):
        if self.extra is None:
            self.extra = _default_mace_extra() if self.name == "mace" else {}


@dataclass
class DataConfig:
    train_path: Optional[str] = None
    val_path: Optional[str] = None
    test_path: Optional[str] = None
    cutoff: float = 4.0
    batch_size: int = 16
    num_workers: int = 0
    val_fraction: float = 0.1
    test_fraction: float = 0.0
    energy_key: str = "energy"
    forces_key: str = "forces"
    stress_key: str = "stress"
    energy_unit: str = "eV"
    length_unit: str = "A"
    head: Optional[str] = None
    replay_path: Optional[str] = None
    replay_head: str = "pt_head"
    replay_samples: Optional[int] = None
    replay_filter: str = "subset"
    replay_pseudolabel: bool = False
    shuffle: bool = True
    pin_memory: bool = True


@dataclass
class OptimConfig:
    lr: float = 1e-3
    weight_decay: float = 0.0
    epochs: int = 100
    energy_weight: float = 1.0
    force_weight: float = 10.0
    stress_weight: float = 0.0
    dipole_weight: float = 0.0
    polarizability_weight: float = 0.0
    charge_weight: float = 0.0
    les_dipole_weight: float = 0.0
    les_charge_weight: float = 0.0
    property_weight: float = 0.0
    reaction_weight: float = 0.0
    reaction_batch_size: int = 16
    scheduler: str = "plateau"
    huber_delta: float = 0.0
    huber_delta_energy: Optional[float] = None
    huber_delta_forces: Optional[float] = None
    huber_delta_stress: Optional[float] = None
    huber_delta_reactions: Optional[float] = None
    optimizer: str = "adam"
    clip_grad: float = 0.0
    ema_decay: float = 0.0
    head_weights: Optional[Dict[str, Dict[str, float]]] = None
    freeze: List[str] = field(default_factory=list)
    train_only: List[str] = field(default_factory=list)
    prior_weight: float = 0.0
    prior_weights: Optional[Dict[str, float]] = None
    loss_weighting: str = "fixed"
    plateau_patience: int = 10
    plateau_factor: float = 0.8
    min_lr: float = 0.0


@dataclass
class TrainerConfig:
    loggers: List[str] = field(default_factory=lambda: ["console"])
    log_every_n_epochs: int = 1
    log_every_n_steps: int = 0
    step_average: str = "batch"
    metrics: List[str] = field(default_factory=lambda: ["mae", "rmse"])
    monitor: str = "val/loss"
    mode: str = "min"
    val_every_n_epochs: int = 1
    save_every_n_epochs: int = 0
    early_stopping_patience: int = 0
    early_stopping_min_delta: float = 0.0
    early_stopping_threshold: Optional[float] = None
    progress_bar: bool = False
    cuda_graph: bool = False
    grad_sync: str = "auto"        # auto / nccl / p2p: how data-parallel gradients are reduced
    graph_headroom: float = 0.05   # padding headroom of a captured step
    #: the hand-written MACE step (energies, forces, loss and gradients without autograd):
    #: "auto" on CUDA when the model and loss are covered, True / False to force it on / off
    fused_step: Any = "auto"


@dataclass
class Config:
    model: ModelConfig = field(default_factory=ModelConfig)
    data: DataConfig = field(default_factory=DataConfig)
    optim: OptimConfig = field(default_factory=OptimConfig)
    trainer: TrainerConfig = field(default_factory=TrainerConfig)
    device: str = "auto"
    seed: int = 1234
    output_dir: str = "runs/exp"
    subtracted_dispersion: Optional[Dict[str, Any]] = None

    def __post_init__(self):
        self.data.cutoff = float(self.model.cutoff)

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)


class IgnoredOptionWarning(UserWarning):
    """A config key that nothing reads."""


# upstream spellings -> (section, key)
TRANSLATIONS = {
    "r_max": ("model", "cutoff"), "num_channels": ("model", "n_features"),
    "num_interactions": ("model", "n_interactions"), "num_radial_basis": ("model", "n_rbf"),
    "num_bessel": ("model", "n_rbf"), "num_layers": ("model", "n_interactions"),
    "max_num_epochs": ("optim", "epochs"), "batch_size": ("data", "batch_size"),
    "E0s": ("model.extra", "atomic_energies"), "atomic_numbers": ("model.extra", "species"),
    "lr": ("optim", "lr"), "energy_weight": ("optim", "energy_weight"),
    "forces_weight": ("optim", "force_weight"), "stress_weight": ("optim", "stress_weight"),
    "l_max": ("model.extra", "l_max"), "model": ("model", "name"),
}


def _coerce(value: str):
    try:
        return ast.literal_eval(value)
    except Exception:
        low = value.lower()
        if low in ("true", "false"):
            return low == "true"
        if low in ("none", "null"):
            return None
        return value


def _set_dotted(d: Dict[str, Any], key: str, value) -> None:
    parts = key.split(".")
    cur = d
    for p in parts[:-1]:
        cur = cur.setdefault(p, {})
    cur[parts[-1]] = value


def _build(cls, data: Dict[str, Any], path: str):
    kw = {}
    names = {f.name: f for f in fields(cls)}
    for k, v in data.items():
        if k not in names:
            warnings.warn(f"config key {path}{k} is not used", IgnoredOptionWarning, stacklevel=3)
            continue
        f = names[k]
        default = f.default_factory() if f.default_factory is not field().default_factory else f.default  # type: ignore
        if is_dataclass(default) and isinstance(v, dict):
            kw[k] = _build(type(default), v, f"{path}{k}.")
        else:
            kw[k] = v
    return cls(**kw)


def from_dict(d: Dict[str, Any], overrides: Optional[Dict[str, Any]] = None) -> Config:
    """A :class:`Config` from a nested dict; top-level upstream keys are translated."""
    d = copy.deepcopy(dict(d or {}))
    for k in list(d):
        if "." in k:
            _set_dotted(d, k, d.pop(k))
    for k in list(d):
        if k in TRANSLATIONS and k not in ("model",) and not isinstance(d[k], dict):
            sec, key = TRANSLATIONS[k]
            v = d.pop(k)
            _set_dotted(d, f"{sec}.{key}", v)
    for k, v in (overrides or {}).items():
        _set_dotted(d, k, v)
    model = d.get("model", {})
    if isinstance(model, str):
        d["model"] = {"name": model}
    elif isinstance(model, dict):
        # a model option that is not a core field is a family option (model.extra), as in the
        # family config files; upstream spellings of the core fields are translated first
        core = {f.name for f in fields(ModelConfig)}
        mod_keys = {"r_max": "cutoff", "num_channels": "n_features", "num_interactions": "n_interactions",
                    "num_radial_basis": "n_rbf", "num_bessel": "n_rbf"}
        folded = {}
        for k in list(model):
            if k in mod_keys and mod_keys[k] not in model:
                model[mod_keys[k]] = model.pop(k)
            elif k not in core:
                folded[k] = model.pop(k)
        if folded:
            model["extra"] = {**folded, **dict(model.get("extra") or {})}
    cfg = _build(Config, d, "")
    if cfg.model.name == "mace":
        base = _default_mace_extra()
        base.update(cfg.model.extra or {})
        cfg.model.extra = base
    cfg.data.cutoff = float(cfg.model.cutoff)
    return cfg


def _compose_defaults(d: Dict[str, Any], base_dir: str) -> Dict[str, Any]:
    """Hydra-style ``defaults``: ``[{model: schnet}, {data: default}, _self_]`` reads
    ``<dir>/model/schnet.yaml`` and ``<dir>/data/default.yaml`` into those sections; the file's
    own keys win when ``_self_`` comes last (the default), the groups' when it comes first."""
    import yaml
    defaults = d.pop("defaults", None)
    if not defaults:
        return d
    self_last = not (defaults and defaults[0] == "_self_")
    groups: Dict[str, Any] = {}
    for item in defaults:
        if item == "_self_" or not isinstance(item, dict):
            continue
        for group, name in item.items():
            with open(os.path.join(base_dir, str(group), f"{name}.yaml")) as f:
                groups[str(group)] = yaml.safe_load(f) or {}
    for group, body in groups.items():
        mine = d.get(group)
        if isinstance(mine, dict) and isinstance(body, dict):
            d[group] = {**body, **mine} if self_last else {**mine, **body}
        elif mine is None or not self_last:
            d[group] = body
    return d


def from_yaml(path: str, overrides: Optional[Dict[str, Any]] = None) -> Config:
    """A run config from a YAML file; a ``defaults`` list composes group files from the same
    directory tree (the shipped ``configs/`` layout: ``model/<family>.yaml``, ``data/*.yaml``)."""
    import yaml
    with open(path) as f:
        d = yaml.safe_load(f) or {}
    d = _compose_defaults(d, os.path.dirname(os.path.abspath(path)))
    return from_dict(d, overrides)


def from_argparse(args) -> Config:
    """``args.config`` (a YAML path, optional) and ``args.set`` (``["a.b=c", ...]``)."""
    overrides = {}
    for item in getattr(args, "set", None) or []:
        k, _, v = item.partition("=")
        overrides[k.strip()] = _coerce(v.strip())
    if getattr(args, "config", None):
        return from_yaml(args.config, overrides)
    return from_dict({}, overrides)


def _plain(node):
    """A nested plain container of a mapping / sequence tree (OmegaConf nodes included)."""
    if isinstance(node, (str, bytes, int, float, bool)) or node is None:
        return node
    if hasattr(node, "items"):
        return {str(k): _plain(v) for k, v in node.items()}
    if isinstance(node, (list, tuple)) or (hasattr(node, "__iter__") and hasattr(node, "__len__")):
        return [_plain(v) for v in node]
    return node


def from_hydra(dict_config) -> Config:
    """A :class:`Config` from a Hydra / OmegaConf ``DictConfig`` (interpolations resolved when
    OmegaConf is installed; any mapping otherwise), through :func:`from_dict`. Parity:
    ``src/xnn/common/config/loaders.py:182``."""
    try:
        from omegaconf import OmegaConf
        container = OmegaConf.to_container(dict_config, resolve=True)
    except (ModuleNotFoundError, ValueError):
        container = _plain(dict_config)
    return from_dict(container)


def apply_overrides(cfg: Config, overrides) -> Config:
    """Apply ``"a.b=c"`` dotted overrides (values parsed as Python literals, else strings) and
    return the new config; an entry without ``=`` is ignored with an
    :class:`IgnoredOptionWarning`. The same syntax as ``--set`` on the command line."""
    parsed = {}
    for item in overrides or []:
        if "=" not in item:
            warnings.warn(f"override {item!r} has no '='", IgnoredOptionWarning, stacklevel=2)
            continue
        k, _, v = item.partition("=")
        parsed[k.strip()] = _coerce(v.strip())
    return from_dict(cfg.to_dict(), parsed)
