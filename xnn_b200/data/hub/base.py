"""Registry of dataset builders and the ``load_dataset`` entry point."""
from __future__ import annotations

from pathlib import Path
from typing import Any, Dict, List, Optional, Union

from .download import default_cache_dir

_REGISTRY: Dict[str, "DatasetBuilder"] = {}


class DatasetBuilder:
    """A named dataset: ``load(split=..., cache_dir=..., **options)`` returns a list of structure
    dicts (``pos``, ``atomic_numbers`` and labels) or a dict of such lists per split."""
    name: str = ""
    description: str = ""

    def load(self, *, split: Optional[str], cache_dir: Path, **kwargs: Any):
        raise NotImplementedError


def register_dataset(builder: DatasetBuilder) -> DatasetBuilder:
    _REGISTRY[builder.name] = builder
    return builder


def get_builder(name: str) -> DatasetBuilder:
    try:
        return _REGISTRY[name]
    except KeyError:
        raise KeyError(f"unknown dataset {name!r}; available: {', '.join(list_datasets())}") from None


def list_datasets() -> List[str]:
    return sorted(_REGISTRY)


def select_split(splits: Dict[str, list], split: Optional[str]):
    if split is None:
        return splits
    if split == "all":
        return [s for part in splits.values() for s in part]
    if split not in splits:
        raise ValueError(f"unknown split {split!r}; use {', '.join(splits)}, 'all' or None")
    return splits[split]


def load_dataset(name: str, *, split: Optional[str] = None, cutoff: Optional[float] = None,
                 cache_dir: Optional[Union[str, Path]] = None, **kwargs: Any):
    """Structures of dataset ``name`` (one split or a dict of splits); with ``cutoff`` wrapped in
    :class:`~xnn_b200.data.AtomicDataset` (neighbour lists built once)."""
    builder = get_builder(name)
    base = Path(cache_dir).expanduser() if cache_dir is not None else default_cache_dir()
    result = builder.load(split=split, cache_dir=base, **kwargs)
    if cutoff is None:
        return result
    from ..dataset import AtomicDataset

    def wrap(items):
        return AtomicDataset(items, cutoff) if items and isinstance(items[0], dict) and "pos" in items[0] else items
    return {k: wrap(v) for k, v in result.items()} if isinstance(result, dict) else wrap(result)
