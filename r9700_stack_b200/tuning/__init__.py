"""Kernel micro-benchmarks and sweeps (graph-free, CUDA-event timed)."""
