"""Benchmarks beyond the flagship training step (bench.py at the repository root)."""
