"""Configuration dataclasses and their loaders."""
from .schema import (Config, DataConfig, IgnoredOptionWarning, ModelConfig, OptimConfig,
                     TrainerConfig, apply_overrides, from_argparse, from_dict, from_hydra, from_yaml)

__all__ = ["Config", "DataConfig", "IgnoredOptionWarning", "ModelConfig", "OptimConfig",
           "TrainerConfig", "apply_overrides", "from_argparse", "from_dict", "from_hydra", "from_yaml"]
