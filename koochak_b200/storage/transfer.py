"""Copy objects between stores: parallel, SHA-256 checked, resumable.

(reference: koochak/storage/transfer.py:42-217)

``copy_objects`` moves bytes between stores; archive, pull, staging and
checkpoint replication build on it. Concurrency defaults come from the
stores' profiles: ``streams`` items at once; an item larger than
``part_bytes`` is read as up to ``range_streams`` parallel byte ranges (kept
in order) and written as one sequential create-only ``put``. A target that
already exists with the expected size is skipped (write-once objects are
complete once visible), so re-running an interrupted copy resumes it; a
different size is refused. Bytes are hashed in flight and a just-written
object whose SHA-256 differs from the expected one is removed and reported.
"""

from __future__ import annotations

import hashlib
import re
import time
from collections import deque
from concurrent.futures import FIRST_COMPLETED, Future, ThreadPoolExecutor, wait
from dataclasses import dataclass
from typing import Callable, Deque, Iterable, Iterator, Optional, Set, Tuple

from .store import Store, profile_of, validate_key

__all__ = ["TransferItem", "TransferReport", "copy_objects"]

ProgressFn = Callable[[int, int, int], None]
_HEX64 = re.compile(r"[0-9a-f]{64}")
_CHUNK = 8 << 20


@dataclass(frozen=True)
class TransferItem:
    source: str
    target: str
    size: Optional[int] = None
    sha256: Optional[str] = None

    def __post_init__(self) -> None:
        validate_key(self.source, "source key")
        validate_key(self.target, "target key")
        if self.size is not None and (type(self.size) is not int or self.size < 0):
            raise ValueError(f"size must be a non-negative integer or None: {self.size!r}")
        if self.sha256 is not None and (not isinstance(self.sha256, str) or not _HEX64.fullmatch(self.sha256)):
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


def _sequential(src: Store, key: str) -> Iterator[bytes]:
    with src.open(key) as fh:
        while True:
            b = fh.read(_CHUNK)
            if not b:
                return
            yield b


def _ranges(src: Store, key: str, size: int, lanes: int, part: int) -> Iterator[bytes]:
    starts = iter(range(0, size, part))
    with ThreadPoolExecutor(max_workers=lanes) as pool:
        q: Deque[Tuple[int, Future]] = deque()

        def more() -> None:
            off = next(starts, None)
            if off is not None:
                n = min(part, size - off)
                q.append((n, pool.submit(src.get, key, off, n)))

        for _ in range(lanes):
            more()
        while q:
            n, fut = q.popleft()
            data = fut.result()
            if len(data) != n:
                raise ValueError(f"{key} is shorter than its expected {size} bytes")
            more()
            yield data


def _copy(src: Store, dst: Store, it: TransferItem, lanes: int, part: int) -> Tuple[bool, int]:
    size = it.size
    if size is None:
        info = src.stat(it.source)
        if info is None:
            raise FileNotFoundError(f"source object does not exist: {it.source}")
        size = info.size
    have = dst.stat(it.target)
    if have is not None:
        if have.size != size:
            raise FileExistsError(f"target {it.target} already exists with {have.size} bytes, expected {size}")
        return False, 0
    chunks = _ranges(src, it.source, size, lanes, part) if lanes > 1 and size > part else _sequential(src, it.source)
    h = hashlib.sha256()
    n = 0

    def hashed() -> Iterator[bytes]:
        nonlocal n
        for c in chunks:
            h.update(c)
            n += len(c)
            yield c

    dst.put(it.target, hashed())
    problem = None
    if n != size:
        problem = f"copied {n} bytes, expected {size}"
    elif it.sha256 is not None and h.hexdigest() != it.sha256:
        problem = "SHA256 does not match the expected digest"
    if problem is not None:
        dst.delete(it.target)  # this call created it
        raise ValueError(f"{it.source} -> {it.target}: {problem}")
    return True, n


def copy_objects(source: Store, target: Store, items: Iterable[TransferItem], *, streams: Optional[int] = None,
                 range_streams: Optional[int] = None, part_bytes: Optional[int] = None,
                 progress: Optional[ProgressFn] = None) -> TransferReport:
    """Copy every item; the first failure stops new work, lets running items finish, and is raised."""

    work = tuple(items)
    if any(not isinstance(i, TransferItem) for i in work):
        raise TypeError("expected TransferItem entries")
    if len({i.target for i in work}) != len(work):
        raise ValueError("transfer items must have unique target keys")
    sp = profile_of(source)
    streams = max(sp.streams, profile_of(target).streams) if streams is None else streams
    range_streams = sp.range_streams if range_streams is None else range_streams
    part_bytes = sp.part_bytes if part_bytes is None else part_bytes
    for name, v in (("streams", streams), ("range_streams", range_streams), ("part_bytes", part_bytes)):
        if type(v) is not int or v < 1:
            raise ValueError(f"{name} must be a positive integer")
    t0 = time.perf_counter()
    copied = skipped = nbytes = 0
    error: Optional[BaseException] = None
    todo = iter(work)
    running: Set[Future] = set()
    with ThreadPoolExecutor(max_workers=streams) as pool:
        def fill() -> None:
            while error is None and len(running) < 2 * streams:
                it = next(todo, None)
                if it is None:
                    return
                running.add(pool.submit(_copy, source, target, it, range_streams, part_bytes))

        fill()
        while running:
            done, _ = wait(running, return_when=FIRST_COMPLETED)
            for fut in done:
                running.discard(fut)
                try:
                    was_copied, n = fut.result()
                except BaseException as exc:
                    error = error or exc
                    continue
                if was_copied:
                    copied += 1
                    nbytes += n
                else:
                    skipped += 1
                if progress is not None:
                    progress(copied + skipped, len(work), nbytes)
            fill()
    if error is not None:
        raise error
    return TransferReport(copied, skipped, nbytes, time.perf_counter() - t0)
