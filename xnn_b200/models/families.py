"""Imports every model family so that their ``@register_model`` decorators run."""
from . import mace, nequip, tensornet  # noqa: F401
