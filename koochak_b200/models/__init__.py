"""Benchmark models built on the native kernels: GPT-2, Llama-style decoder, ViT, MLP."""

from .gpt2 import GPT2, GPT2Config  # noqa: F401
from .llama import Llama, LlamaConfig  # noqa: F401
from .mlp import MLP  # noqa: F401
from .vit import ViT, ViTConfig  # noqa: F401
