"""Directory-level checkpoint lookup (reference: koochak/storage/fs.py:11-53)."""

from __future__ import annotations

import os
import re
from typing import List, Optional

import torch

from .naming import DEFAULT_STEP_PATTERN
from .pruning import _extract_step

__all__ = ["mkdir_p", "latest", "best"]


def mkdir_p(path: str) -> None:
    os.makedirs(path, exist_ok=True)


def _step_files(directory: str, pattern: str) -> List[str]:
    if not os.path.isdir(directory):
        return []
    rx = re.compile(pattern)
    found = [os.path.join(directory, f) for f in os.listdir(directory) if rx.search(f)]
    found.sort(key=lambda p: _extract_step(os.path.basename(p), rx))
    return found


def latest(directory: str, pattern: str = DEFAULT_STEP_PATTERN) -> Optional[str]:
    """``latest.pt`` when present, else the highest-step match."""

    link = os.path.join(directory, "latest.pt")
    if os.path.exists(link):
        return link
    files = _step_files(directory, pattern)
    return files[-1] if files else None


def best(directory: str, key: str = "val_loss", pattern: str = DEFAULT_STEP_PATTERN) -> Optional[str]:
    """The checkpoint whose ``metrics[key]`` is smallest."""

    winner, best_val = None, float("inf")
    for path in _step_files(directory, pattern):
        try:
            ckpt = torch.load(path, weights_only=False, map_location="cpu")
        except (OSError, RuntimeError, EOFError):
            continue
        metrics = ckpt.get("metrics") or {}
        if key not in metrics:
            continue
        try:
            val = float(metrics[key])
        except (TypeError, ValueError):
            continue
        if val < best_val:
            winner, best_val = path, val
    return winner
