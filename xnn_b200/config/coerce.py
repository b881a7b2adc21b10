"""Coercion of config values copied from upstream YAML files (``src/xnn/common/config/coerce.py``)."""
from __future__ import annotations

import ast
from typing import List, Optional


def coerce_species(value, default: Optional[List[int]] = None) -> List[int]:
    if value is None:
        return list(default or [])
    if isinstance(value, str):
        value = ast.literal_eval(value)
    return [int(z) for z in value]


def coerce_per_species(value, species: List[int], what: str = "values"):
    """A list aligned with ``species`` from a list, a ``{Z: value}`` dict or their string forms."""
    if value is None:
        return None
    if isinstance(value, str):
        value = ast.literal_eval(value)
    if isinstance(value, dict):
        missing = [z for z in species if z not in value and str(z) not in value]
        if missing:
            raise ValueError(f"{what}: no value for species {missing}")
        return [float(value[z] if z in value else value[str(z)]) for z in species]
    value = [float(v) for v in value]
    if len(value) != len(species):
        raise ValueError(f"{what}: {len(value)} values for {len(species)} species")
    return value
