"""Utilities: kernel micro-benchmarks, timing helpers."""
