"""Score checkpoints on labelled structures (energy / force / stress errors)."""
from .runner import error_report, evaluate_structures, format_report, run_benchmark

__all__ = ["error_report", "evaluate_structures", "format_report", "run_benchmark"]
