"""Deployment: MD drivers, calculators, exporters."""
