"""Checkpoint names and aliases (reference: koochak/storage/naming.py:12-68)."""

from __future__ import annotations

import os
import re
from typing import Iterable, List, Optional, Pattern

__all__ = ["DEFAULT_STEP_PATTERN", "parse_step_from_name", "parse_step_from_path", "make_checkpoint_aliases"]

DEFAULT_STEP_PATTERN: str = r"step(\d+)\.pt$"
_DEFAULT_RX: Pattern[str] = re.compile(DEFAULT_STEP_PATTERN)


def _step_from_match(match: "re.Match[str]") -> Optional[int]:
    """Integer of the last capture group that parses as one."""

    for group in reversed(match.groups()):
        if group is None:
            continue
        try:
            return int(group)
        except ValueError:
            pass
    return None


def parse_step_from_name(name: str, pattern: str = DEFAULT_STEP_PATTERN) -> Optional[int]:
    rx = _DEFAULT_RX if pattern == DEFAULT_STEP_PATTERN else re.compile(pattern)
    m = rx.search(name)
    return _step_from_match(m) if m else None


def parse_step_from_path(path: str, pattern: str = DEFAULT_STEP_PATTERN) -> Optional[int]:
    return parse_step_from_name(os.path.basename(path), pattern)


def make_checkpoint_aliases(step: Optional[int], *, include_latest: bool = True,
                            best_keys: Optional[Iterable[str]] = None) -> List[str]:
    """``["latest", "step-N", "best", "best-<key>"...]`` as applicable."""

    out: List[str] = ["latest"] if include_latest else []
    if step is not None:
        out.append(f"step-{step}")
    keys = list(best_keys or [])
    if keys:
        out.append("best")
        out.extend(f"best-{k}" for k in keys)
    return out
