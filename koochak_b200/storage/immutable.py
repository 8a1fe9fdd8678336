"""Immutable regular files on shared storage, race-checked.

(reference: koochak/storage/immutable.py:25-165)

``write_immutable_file`` publishes bytes under a name that never gets
replaced: the bytes go to a private temporary file in the same directory,
are fsynced, and are hard-linked into place (``link`` fails if the name
exists). If the name already exists with identical bytes the call succeeds
without writing (idempotent re-publication); different bytes raise
``FileExistsError``.

``read_stable_regular_file`` reads a non-symlink regular file and checks,
with ``fstat`` before and after and ``lstat`` of the name, that neither the
file's identity nor its size / mtime / ctime moved while reading. The one
change tolerated (and re-read) is the publisher dropping its temporary hard
link, which lowers the link count and moves ctime but nothing else.
"""

from __future__ import annotations

import os
import stat
import tempfile
from pathlib import Path
from typing import Tuple

__all__ = ["read_stable_regular_file", "write_immutable_file"]

_NOFOLLOW = os.O_RDONLY | getattr(os, "O_CLOEXEC", 0) | getattr(os, "O_NOFOLLOW", 0)


def _ident(st: os.stat_result) -> Tuple[int, int]:
    return st.st_dev, st.st_ino


def _content_key(st: os.stat_result) -> Tuple[int, int, int]:
    return st.st_size, st.st_mtime_ns, st.st_ctime_ns


def _only_link_dropped(a: os.stat_result, b: os.stat_result) -> bool:
    return b.st_nlink < a.st_nlink and (a.st_size, a.st_mtime_ns, a.st_mode) == (b.st_size, b.st_mtime_ns, b.st_mode)


def _read_fd(fd: int) -> bytes:
    parts = []
    while True:
        chunk = os.read(fd, 1 << 20)
        if not chunk:
            return b"".join(parts)
        parts.append(chunk)


def _read_checked(target: str, err) -> Tuple[bytes, os.stat_result, bool]:
    """Return (bytes, final stat, stable) for one read of ``target``; raise ``err`` on identity changes."""

    fd = os.open(target, _NOFOLLOW)
    try:
        before = os.fstat(fd)
        if not stat.S_ISREG(before.st_mode):
            raise err(f"not a regular file: {target}")
        data = _read_fd(fd)
        after = os.fstat(fd)
    finally:
        os.close(fd)
    try:
        now = os.lstat(target)
    except FileNotFoundError as exc:
        raise err(f"file was replaced while reading: {target}") from exc
    if not (_ident(before) == _ident(after) == _ident(now)) or not stat.S_ISREG(now.st_mode):
        raise err(f"file changed while reading: {target}")
    if _content_key(before) == _content_key(after):
        return data, after, True
    if _only_link_dropped(before, after):
        return data, after, False  # re-read
    raise err(f"file changed while reading: {target}")


def read_stable_regular_file(filename: str | os.PathLike) -> bytes:
    target = os.fspath(filename)
    for _ in range(3):
        data, _st, stable = _read_checked(target, ValueError)
        if stable:
            return data
    raise ValueError(f"file changed while reading: {target}")


def _accept_existing(target: Path, content: bytes, mode: int) -> bool:
    for _ in range(3):
        try:
            data, st, stable = _read_checked(str(target), FileExistsError)
        except OSError as exc:
            if isinstance(exc, FileExistsError):
                raise
            raise FileExistsError(f"refusing non-regular or unstable immutable artifact: {target}") from exc
        if not stable:
            continue
        if data != content:
            raise FileExistsError(f"refusing to replace different artifact: {target}")
        if stat.S_IMODE(st.st_mode) != mode:
            os.chmod(target, mode)  # the name was just verified to be a regular file
        return False
    raise FileExistsError(f"immutable artifact changed while reading: {target}")


def write_immutable_file(filename: str | os.PathLike, content: bytes, *, mode: int = 0o444) -> bool:
    """Publish ``content`` at ``filename`` without ever replacing it; True if this call created it."""

    target = Path(filename)
    target.parent.mkdir(parents=True, exist_ok=True)
    if os.path.lexists(target):
        return _accept_existing(target, content, mode)
    fd, tmp = tempfile.mkstemp(prefix=f".{target.name}.", dir=target.parent)
    try:
        with os.fdopen(fd, "wb") as fh:
            fh.write(content)
            fh.flush()
            os.fsync(fh.fileno())
        os.chmod(tmp, mode)
        try:
            os.link(tmp, target, follow_symlinks=False)
        except FileExistsError:
            return _accept_existing(target, content, mode)
        dfd = os.open(target.parent, os.O_RDONLY)
        try:
            os.fsync(dfd)
        finally:
            os.close(dfd)
        return True
    finally:
        try:
            os.unlink(tmp)
        except FileNotFoundError:
            pass
