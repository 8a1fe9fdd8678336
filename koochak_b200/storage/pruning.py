"""Keep-last-k pruning of step-numbered files (reference: koochak/storage/pruning.py:10-49)."""

from __future__ import annotations

import os
import re
from typing import List

from .naming import _step_from_match

__all__ = ["prune_keep_last_k"]


def _extract_step(name: str, pattern: "re.Pattern[str]") -> int:
    m = pattern.search(name)
    step = _step_from_match(m) if m else None
    return -1 if step is None else step


def prune_keep_last_k(directory: str, pattern: str, k: int, *, companion_suffixes: tuple[str, ...] = ()) -> None:
    """Delete all but the ``k`` highest-step matches (and their sidecars); best-effort."""

    if k <= 0 or not os.path.isdir(directory):
        return
    rx = re.compile(pattern)
    files: List[str] = [os.path.join(directory, f) for f in os.listdir(directory) if rx.search(f)]
    if len(files) <= k:
        return
    files.sort(key=lambda p: _extract_step(os.path.basename(p), rx))
    for path in files[:-k]:
        try:
            os.remove(path)
        except OSError:
            continue
        for suffix in companion_suffixes:
            try:
                os.remove(path + suffix)
            except OSError:
                pass
