"""Benchmark models built on the native kernels: GPT-2, Llama-style decoder, ViT, MLP."""

from .gpt2 import GPT2, GPT2Config  # noqa: F401
