"""Imports every model family so that their ``@register_model`` decorators run."""
from . import d3, mace, nequip, tensornet  # noqa: F401
