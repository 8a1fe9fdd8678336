"""GPU health monitoring (read-only nvidia-smi queries) and Slurm recovery."""

from .gpu import GpuHealthFailure, GpuHealthSample, GpuHealthWatchdog, evaluate_sample, summarize_failures_for_stdout

__all__ = ["GpuHealthFailure", "GpuHealthSample", "GpuHealthWatchdog", "evaluate_sample",
           "summarize_failures_for_stdout"]
