"""Benchmarks: op sweeps and serving traces."""
