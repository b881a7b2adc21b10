"""Dataset hub: named dataset builders behind one ``load_dataset`` call (registry, cached and
MD5-checked downloads that respect ``XNN_B200_OFFLINE``, unit conversion, fixed splits).

    from xnn_b200.data.hub import load_dataset, list_datasets
    train = load_dataset("rmd17", molecule="ethanol", split="train", cutoff=5.0)

The same call shapes as the reference hub (``src/xnn/common/data/hub/base.py:20-160``).
"""
from .base import DatasetBuilder, get_builder, list_datasets, load_dataset, register_dataset  # noqa: F401
from . import builders, gmtkn55, more, qm9  # noqa: F401  (registers the builders)
