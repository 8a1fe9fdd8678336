"""Finding checkpoints in a plain directory: the newest, or the best by a logged metric.

(behaviour of reference koochak/storage/fs.py:11-53)
"""

from __future__ import annotations

import os
import re
from typing import Iterator, List, Optional, Tuple

import torch

from .naming import DEFAULT_STEP_PATTERN
from .pruning import _extract_step

__all__ = ["mkdir_p", "latest", "best"]


def mkdir_p(path: str) -> None:
    os.makedirs(path, exist_ok=True)


def _matching(directory: str, pattern: str) -> List[str]:
    """Paths in ``directory`` whose names match ``pattern``, in increasing step order."""

    if not os.path.isdir(directory):
        return []
    rx = re.compile(pattern)
    names = sorted((n for n in os.listdir(directory) if rx.search(n)), key=lambda n: _extract_step(n, rx))
    return [os.path.join(directory, n) for n in names]


def latest(directory: str, pattern: str = DEFAULT_STEP_PATTERN) -> Optional[str]:
    """``latest.pt`` when it exists, else the matching file with the highest step."""

    alias = os.path.join(directory, "latest.pt")
    if os.path.exists(alias):
        return alias
    found = _matching(directory, pattern)
    return found[-1] if found else None


def _scored(paths: List[str], key: str) -> Iterator[Tuple[float, str]]:
    for path in paths:
        try:
            metrics = torch.load(path, weights_only=False, map_location="cpu").get("metrics") or {}
            yield float(metrics[key]), path
        except (OSError, RuntimeError, EOFError, KeyError, TypeError, ValueError):
            continue  # unreadable, or no usable value of the metric


def best(directory: str, key: str = "val_loss", pattern: str = DEFAULT_STEP_PATTERN) -> Optional[str]:
    """The matching checkpoint with the smallest ``metrics[key]`` (the earliest on ties)."""

    winner: Optional[Tuple[float, str]] = None
    for score, path in _scored(_matching(directory, pattern), key):
        if winner is None or score < winner[0]:
            winner = (score, path)
    return winner[1] if winner else None
