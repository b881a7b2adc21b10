"""Command line: ``python -m xnn_b200 {train,benchmark,export,mdi,models}``."""
from .main import main

__all__ = ["main"]
