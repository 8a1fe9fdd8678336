"""Atomic small-file writes (reference: koochak/storage/atomic.py:9-34)."""

from __future__ import annotations

import os
import tempfile

__all__ = ["atomic_write"]


def _fsync_directory(directory: str) -> None:
    fd = os.open(directory, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def atomic_write(path: str, data: bytes, tmp_suffix: str = ".tmp") -> None:
    """Write ``data`` to a temp file in the same directory, fsync, then rename over ``path``."""

    directory = os.path.dirname(os.path.abspath(path)) or "."
    os.makedirs(directory, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=tmp_suffix, dir=directory)
    try:
        with os.fdopen(fd, "wb") as fh:
            fh.write(data)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, path)
        _fsync_directory(directory)
    finally:
        if os.path.exists(tmp):
            try:
                os.remove(tmp)
            except OSError:
                pass
