"""Kernel- and step-level benchmarks (CUDA-event timed)."""
