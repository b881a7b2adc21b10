"""Imports every model family so that their ``@register_model`` decorators run."""
from . import d3, d4, mace, nequip, painn, qet, schnet, tensornet  # noqa: F401
