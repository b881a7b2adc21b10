"""Model runtime (contract, registry, forces/stress) and the model families."""
from .base import GNNPotential, InteratomicPotential
from .outputs import ForceStressOutput
from .registry import MODELS, build_model, get_model_class, list_models, prepare_model, register_model

__all__ = ["ForceStressOutput", "GNNPotential", "InteratomicPotential", "MODELS", "build_model",
           "get_model_class", "list_models", "prepare_model", "register_model"]
