"""MNIST-shaped MLP (784 -> 256 ReLU -> 10), the plumbing workload of the CPU benchmark.

Plain PyTorch: at this size every kernel launch costs more than its math, so
the model is only used to exercise the runtime (data parallel over gloo,
checkpoint save / resume) and runs on any device.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["MLP"]


class MLP(nn.Module):
    def __init__(self, in_dim: int = 28 * 28, hidden: int = 256, classes: int = 10) -> None:
        super().__init__()
        self.fc1 = nn.Linear(in_dim, hidden)
        self.fc2 = nn.Linear(hidden, classes)

    def forward(self, x: torch.Tensor, labels: torch.Tensor | None = None):
        logits = self.fc2(F.relu(self.fc1(x.flatten(1))))
        return logits if labels is None else F.cross_entropy(logits, labels)
