"""Filesystem path normalisation (reference: koochak/utils/paths.py:6-10)."""

from __future__ import annotations

import os

__all__ = ["canonical_dir"]


def canonical_dir(path: str) -> str:
    """Absolute path with ``~`` expanded; used for every directory setting."""

    return os.path.abspath(os.path.expanduser(os.fspath(path)))
