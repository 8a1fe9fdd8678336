"""Copying objects between stores: parallel, SHA-256 checked, resumable.

(behaviour of reference koochak/storage/transfer.py:42-217)

``copy_objects`` is the byte mover under archive, pull, staging and
checkpoint replication. Concurrency defaults come from the stores' profiles:
up to ``streams`` objects at a time; an object larger than ``part_bytes`` is
read as up to ``range_streams`` concurrent byte ranges (consumed in order)
and written as one sequential create-only ``put``.

Resumability: a target that already exists with the expected size is
skipped, because a write-once object is complete once visible; a different
size is refused. Integrity: bytes are hashed while they stream, and a
freshly written object whose size or SHA-256 is wrong is deleted and
reported.
"""

from __future__ import annotations

import hashlib
import re
import time
from collections import deque
from concurrent.futures import FIRST_COMPLETED, Future, ThreadPoolExecutor, wait
from dataclasses import dataclass
from typing import Callable, Deque, Iterable, Iterator, List, Optional, Set, Tuple

from .store import Store, profile_of, validate_key

__all__ = ["TransferItem", "TransferReport", "copy_objects"]

ProgressFn = Callable[[int, int, int], None]
_SHA256_HEX = re.compile(r"[0-9a-f]{64}")
_READ_BLOCK = 8 << 20


@dataclass(frozen=True)
class TransferItem:
    source: str
    target: str
    size: Optional[int] = None
    sha256: Optional[str] = None

    def __post_init__(self) -> None:
        validate_key(self.source, "source key")
        validate_key(self.target, "target key")
        if self.size is not None and not (type(self.size) is int and self.size >= 0):
            raise ValueError(f"size must be a non-negative integer or None: {self.size!r}")
        if self.sha256 is not None and not (isinstance(self.sha256, str) and _SHA256_HEX.fullmatch(self.sha256)):
            raise ValueError(f"sha256 must be 64 lowercase hex characters: {self.sha256!r}")


@dataclass(frozen=True)
class TransferReport:
    copied: int
    skipped: int
    bytes_copied: int
    seconds: float

    @property
    def mb_s(self) -> float:
        return self.bytes_copied / max(self.seconds, 1e-9) / 1e6


class _Copier:
    """Copies one object at a time from ``src`` to ``dst`` (thread-safe: no shared state)."""

    def __init__(self, src: Store, dst: Store, lanes: int, part: int) -> None:
        self.src, self.dst, self.lanes, self.part = src, dst, lanes, part

    def _whole(self, key: str) -> Iterator[bytes]:
        with self.src.open(key) as fh:
            yield from iter(lambda: fh.read(_READ_BLOCK), b"")

    def _in_ranges(self, key: str, size: int) -> Iterator[bytes]:
        offsets = list(range(0, size, self.part))
        with ThreadPoolExecutor(max_workers=self.lanes) as pool:
            window: Deque[Tuple[int, Future]] = deque()
            for off in offsets:
                want = min(self.part, size - off)
                window.append((want, pool.submit(self.src.get, key, off, want)))
                if len(window) < self.lanes:
                    continue
                yield self._take(window, key, size)
            while window:
                yield self._take(window, key, size)

    @staticmethod
    def _take(window: Deque[Tuple[int, Future]], key: str, size: int) -> bytes:
        want, pending = window.popleft()
        data = pending.result()
        if len(data) != want:
            raise ValueError(f"{key} is shorter than its expected {size} bytes")
        return data

    def copy(self, item: TransferItem) -> Tuple[bool, int]:
        """(copied?, bytes); a complete existing target is left alone."""

        size = item.size
        if size is None:
            info = self.src.stat(item.source)
            if info is None:
                raise FileNotFoundError(f"source object does not exist: {item.source}")
            size = info.size
        existing = self.dst.stat(item.target)
        if existing is not None:
            if existing.size != size:
                raise FileExistsError(f"target {item.target} already exists with {existing.size} bytes, "
                                      f"expected {size}")
            return False, 0
        stream = (self._in_ranges(item.source, size) if self.lanes > 1 and size > self.part
                  else self._whole(item.source))
        digest = hashlib.sha256()
        count = [0]

        def observed() -> Iterator[bytes]:
            for piece in stream:
                digest.update(piece)
                count[0] += len(piece)
                yield piece

        self.dst.put(item.target, observed())
        wrong = None
        if count[0] != size:
            wrong = f"copied {count[0]} bytes, expected {size}"
        elif item.sha256 is not None and digest.hexdigest() != item.sha256:
            wrong = "SHA256 does not match the expected digest"
        if wrong:
            self.dst.delete(item.target)  # written by this call
            raise ValueError(f"{item.source} -> {item.target}: {wrong}")
        return True, count[0]


def _positive(name: str, value: object) -> int:
    if type(value) is not int or value < 1:
        raise ValueError(f"{name} must be a positive integer")
    return value


def copy_objects(source: Store, target: Store, items: Iterable[TransferItem], *, streams: Optional[int] = None,
                 range_streams: Optional[int] = None, part_bytes: Optional[int] = None,
                 progress: Optional[ProgressFn] = None) -> TransferReport:
    """Copy every item. The first failure stops new work; items already running finish; it is raised."""

    todo: List[TransferItem] = list(items)
    if not all(isinstance(i, TransferItem) for i in todo):
        raise TypeError("expected TransferItem entries")
    if len({i.target for i in todo}) != len(todo):
        raise ValueError("transfer items must have unique target keys")
    src_profile = profile_of(source)
    streams = _positive("streams", max(src_profile.streams, profile_of(target).streams) if streams is None
                        else streams)
    lanes = _positive("range_streams", src_profile.range_streams if range_streams is None else range_streams)
    part = _positive("part_bytes", src_profile.part_bytes if part_bytes is None else part_bytes)
    copier = _Copier(source, target, lanes, part)
    started = time.perf_counter()
    copied = skipped = moved = 0
    failure: Optional[BaseException] = None
    queue = iter(todo)
    active: Set[Future] = set()
    with ThreadPoolExecutor(max_workers=streams) as pool:
        while True:
            while failure is None and len(active) < 2 * streams:
                nxt = next(queue, None)
                if nxt is None:
                    break
                active.add(pool.submit(copier.copy, nxt))
            if not active:
                break
            finished, active = wait(active, return_when=FIRST_COMPLETED)
            for fut in finished:
                try:
                    did_copy, nbytes = fut.result()
                except BaseException as exc:
                    failure = failure or exc
                    continue
                copied, skipped, moved = copied + did_copy, skipped + (not did_copy), moved + nbytes
                if progress is not None:
                    progress(copied + skipped, len(todo), moved)
    if failure is not None:
        raise failure
    return TransferReport(copied, skipped, moved, time.perf_counter() - started)
