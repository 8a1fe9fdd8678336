"""Stream the groups of a packed collection to data-loading workers.

(behaviour of reference koochak/data/packed.py:77-412)

An archive written with a groups table (``python -m koochak_b200.data archive
--groups``) keeps every file one training record needs contiguous inside one
pack. This module reads it the way object storage likes: few, large,
sequential requests.

* ``PackedGroups`` indexes the file table by group; a group belongs to the
  pack holding its first file. ``plan(num_owners=...)`` deals whole packs to
  the job's workers with ``plan_shards`` (groups as the records), so workers
  own disjoint groups and every rank computes the same plan.
* ``GroupStream`` is one worker's endless stream of ``LoadedGroup``: pass ``p``
  orders the worker's packs by ``sha256(seed, p, pack key)``, fetches whole
  packs ahead in background threads (``prefetch``), verifies each against the
  manifest and yields the groups of each window of ``window`` packs in a
  seeded shuffle. Passes run back to back inside one stream (ranks never run
  dry at different times); ``start`` skips groups for resumption without
  reading the skipped packs.
* ``read_files`` reads chosen files on their own (one open per pack) and
  ``PackCache`` keeps recent packs in memory up to a byte budget.
"""

from __future__ import annotations

import hashlib
import itertools
import random
import threading
import time
from collections import OrderedDict, deque
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Callable, Deque, Dict, Iterator, List, Mapping, Optional, Sequence, Tuple

from ..storage.collection import (Collection, FileEntry, PackRange, load_collection, object_key, pack_ranges,
                                  read_pack_range, read_pack_ranges)
from ..storage.store import Store
from .shards import Shard, plan_shards

__all__ = ["GroupInfo", "GroupStream", "LoadedGroup", "PackCache", "PackedGroups"]


@dataclass(frozen=True)
class GroupInfo:
    name: str
    files: Tuple[FileEntry, ...]
    pack: Optional[int]
    size_bytes: int


@dataclass(frozen=True)
class LoadedGroup:
    name: str
    files: Mapping[str, bytes]
    entries: Mapping[str, FileEntry]


def _hash_order(seed: int, epoch: int, key: str) -> bytes:
    return hashlib.sha256(f"{seed}\x00{epoch}\x00{key}".encode("utf-8")).digest()


def _check(data: bytes, e: FileEntry, verify: bool) -> bytes:
    if len(data) != e.size or (verify and hashlib.sha256(data).hexdigest() != e.sha256):
        raise ValueError(f"{e.path} does not match its file-table size and SHA256")
    return data


def _index_groups(collection: Collection) -> Tuple[Dict[str, GroupInfo], Dict[int, Tuple[str, ...]]]:
    """Groups by name (files in pack/offset order) and, per pack, the groups that start in it."""

    members: Dict[str, List[FileEntry]] = {}
    for e in collection.files:
        members.setdefault(e.group, []).append(e)
    infos: Dict[str, GroupInfo] = {}
    for name, entries in members.items():
        entries.sort(key=lambda x: (x.pack is None, x.pack or 0, x.offset or 0, x.path))
        infos[name] = GroupInfo(name, tuple(entries), entries[0].pack, sum(x.size for x in entries))
    unpacked = sorted(n for n, g in infos.items() if g.pack is None)
    if unpacked:
        raise ValueError(f"{len(unpacked)} groups have no packed file (e.g. {unpacked[:3]}); archive with "
                         "--object-bytes at least as large as --pack-bytes")
    starting: Dict[int, List[str]] = {}
    for name, g in infos.items():
        starting.setdefault(g.pack, []).append(name)  # type: ignore[arg-type]
    per_pack = {p: tuple(sorted(names, key=lambda n: infos[n].files[0].offset or 0)) for p, names in starting.items()}
    return infos, per_pack


def _loaded(name: str, files: Dict[str, bytes], info: GroupInfo) -> LoadedGroup:
    return LoadedGroup(name, MappingProxyType(files), MappingProxyType({e.path: e for e in info.files}))


class PackedGroups:
    def __init__(self, collection: Collection) -> None:
        if not isinstance(collection, Collection):
            raise TypeError("PackedGroups needs a Collection")
        if collection.layout != "packed":
            raise ValueError("PackedGroups needs a collection with the 'packed' layout")
        self.collection = collection
        infos, per_pack = _index_groups(collection)
        self.groups: Mapping[str, GroupInfo] = MappingProxyType(infos)
        self.pack_groups: Mapping[int, Tuple[str, ...]] = MappingProxyType(per_pack)

    @classmethod
    def load(cls, store: Store) -> "PackedGroups":
        return cls(load_collection(store))

    def load_group(self, store: Store, name: str, *, verify: bool = True) -> LoadedGroup:
        """One ranged read per pack the group touches (usually one), objects read whole."""

        info = self.groups[name]
        packed = [e for e in info.files if e.pack is not None]
        # One read per pack: the range from the group's first to its last byte there.
        spans = pack_ranges(packed, self.collection.packs, merge_gap=1 << 62, max_range=1 << 62)
        files: Dict[str, bytes] = {}
        for part in spans:
            files.update(read_pack_range(store, part, verify=verify))
        for e in info.files:
            if e.pack is None:
                files[e.path] = _check(store.get(object_key(e.path)), e, verify)
        return _loaded(name, files, info)

    def read_files(self, store: Store, entries: Sequence[FileEntry], *, verify: bool = True, streams: int = 16,
                   merge_gap: int = 64 * 1024, max_range: int = 16 << 20) -> Dict[str, bytes]:
        """The chosen files, read with one open per pack (ranges merged) and in parallel across packs."""

        wanted = {e.path: e for e in entries}
        by_pack: Dict[str, List[PackRange]] = {}
        for part in pack_ranges([e for e in wanted.values() if e.pack is not None], self.collection.packs,
                                merge_gap=merge_gap, max_range=max_range):
            by_pack.setdefault(part.pack.key, []).append(part)
        tasks: List[Callable[[], Dict[str, bytes]]] = [
            (lambda parts=parts: read_pack_ranges(store, parts, verify=verify)) for parts in by_pack.values()]
        tasks += [(lambda e=e: {e.path: _check(store.get(e.object), e, verify)})
                  for e in wanted.values() if e.pack is None]
        found: Dict[str, bytes] = {}
        if len(tasks) > 1 and streams > 1:
            with ThreadPoolExecutor(max_workers=min(streams, len(tasks))) as pool:
                for part in pool.map(lambda task: task(), tasks):
                    found.update(part)
        else:
            for task in tasks:
                found.update(task())
        return found

    def plan(self, *, num_owners: int, seed: int = 0,
             select: Optional[Callable[[str], bool]] = None) -> Tuple[Tuple[int, ...], ...]:
        """Deal whole packs to ``num_owners`` workers with ``plan_shards`` (a pack's selected groups are its records)."""

        as_shards = []
        for p in sorted(self.pack_groups):
            n = sum(1 for g in self.pack_groups[p] if select is None or select(g))
            if n:
                pe = self.collection.packs[p]
                as_shards.append(Shard(pe.key, pe.size, pe.sha256, n))
        if not as_shards:
            raise ValueError("no pack holds a selected group")
        index_of = {pe.key: i for i, pe in enumerate(self.collection.packs)}
        hands = plan_shards(as_shards, num_workers=num_owners, seed=seed)
        return tuple(tuple(sorted(index_of[sh.key] for sh in hand)) for hand in hands)


@dataclass
class PackCache:
    """Recently fetched packs up to ``max_bytes`` (least recently used out); thread-safe."""

    max_bytes: int
    hits: int = 0
    _packs: "OrderedDict[int, bytes]" = field(default_factory=OrderedDict)
    _bytes: int = 0
    _lock: threading.Lock = field(default_factory=threading.Lock)

    def __post_init__(self) -> None:
        if type(self.max_bytes) is not int or self.max_bytes < 0:
            raise ValueError("max_bytes must be a non-negative integer")

    def get(self, pack: int) -> Optional[bytes]:
        with self._lock:
            data = self._packs.get(pack)
            if data is not None:
                self._packs.move_to_end(pack)
                self.hits += 1
            return data

    def put(self, pack: int, data: bytes) -> None:
        with self._lock:
            if len(data) > self.max_bytes or pack in self._packs:
                return
            self._packs[pack] = data
            self._bytes += len(data)
            while self._bytes > self.max_bytes:
                self._bytes -= len(self._packs.popitem(last=False)[1])


class GroupStream:
    """One worker's endless stream of its groups, pass after pass (see the module notes)."""

    def __init__(self, store: Store, groups: PackedGroups, packs: Sequence[int], *,
                 select: Optional[Callable[[str], bool]] = None, seed: int = 0, window: int = 2, prefetch: int = 2,
                 start: int = 0, verify: bool = True, cache: Optional[PackCache] = None, retries: int = 0,
                 retry_seconds: float = 5.0) -> None:
        for what, value, least in (("window", window, 1), ("prefetch", prefetch, 0), ("start", start, 0),
                                   ("retries", retries, 0)):
            if type(value) is not int or value < least:
                raise ValueError(f"{what} must be an integer >= {least}")
        self.store, self.groups, self.select, self.seed = store, groups, select, seed
        self.window, self.prefetch, self.start, self.verify = window, prefetch, start, verify
        self.cache, self.retries, self.retry_seconds = cache, retries, retry_seconds
        self.selected = {p: tuple(g for g in groups.pack_groups.get(p, ()) if select is None or select(g))
                         for p in packs}
        self.packs = tuple(p for p in sorted(set(packs)) if self.selected[p])
        if not self.packs:
            raise ValueError("this worker owns no selected group")
        self.groups_per_pass = sum(len(self.selected[p]) for p in self.packs)
        self.stats = {"packs_fetched": 0, "bytes_fetched": 0, "fetch_seconds": 0.0, "wait_seconds": 0.0,
                      "cache_hits": 0, "retries": 0}

    # ---------------------------------------------------------------- fetching whole packs
    def _get_with_retries(self, key: str) -> bytes:
        for attempt in range(self.retries + 1):
            try:
                return self.store.get(key)
            except OSError:
                if attempt == self.retries:
                    raise
                self.stats["retries"] += 1
                time.sleep(self.retry_seconds)
        raise AssertionError("unreachable")

    def _fetch(self, p: int) -> bytes:
        cached = self.cache.get(p) if self.cache is not None else None
        if cached is not None:
            self.stats["cache_hits"] += 1
            return cached
        entry = self.groups.collection.packs[p]
        began = time.perf_counter()
        data = self._get_with_retries(entry.key)
        self.stats["fetch_seconds"] += time.perf_counter() - began
        if len(data) != entry.size or (self.verify and hashlib.sha256(data).hexdigest() != entry.sha256):
            raise ValueError(f"{entry.key} does not match its manifest size and SHA256")
        self.stats["packs_fetched"] += 1
        self.stats["bytes_fetched"] += len(data)
        if self.cache is not None:
            self.cache.put(p, data)
        return data

    def _materialize(self, name: str, loaded: Mapping[int, bytes]) -> LoadedGroup:
        info = self.groups.groups[name]
        files: Dict[str, bytes] = {}
        for e in info.files:
            if e.pack in loaded:  # its pack was verified whole
                files[e.path] = loaded[e.pack][e.offset:e.offset + e.size]
            elif e.pack is not None:
                key = self.groups.collection.packs[e.pack].key
                files[e.path] = _check(self.store.get(key, e.offset, e.size), e, self.verify)
            else:
                files[e.path] = _check(self.store.get(object_key(e.path)), e, self.verify)
        return _loaded(name, files, info)

    # ---------------------------------------------------------------- order
    def _windows(self, epoch: int) -> List[Tuple[int, ...]]:
        keys = self.groups.collection.packs
        order = sorted(self.packs, key=lambda p: _hash_order(self.seed, epoch, keys[p].key))
        return [tuple(order[i:i + self.window]) for i in range(0, len(order), self.window)]

    def _shuffled(self, epoch: int, number: int, window: Sequence[int]) -> List[str]:
        names = [g for p in window for g in self.selected[p]]
        random.Random(_hash_order(self.seed, epoch, f"window-{number}")).shuffle(names)
        return names

    def _schedule(self) -> Iterator[Tuple[int, int, Tuple[int, ...], int]]:
        """(pass, window number, packs, groups to skip) forever; ``start`` skips whole windows unread."""

        skip = self.start
        for epoch in itertools.count():
            for number, window in enumerate(self._windows(epoch)):
                size = sum(len(self.selected[p]) for p in window)
                if skip >= size:
                    skip -= size
                    continue
                yield epoch, number, window, skip
                skip = 0

    def __iter__(self) -> Iterator[LoadedGroup]:
        plan = self._schedule()
        pool = ThreadPoolExecutor(max_workers=max(1, self.prefetch))
        queued: Deque[Tuple[int, int, Tuple[int, ...], int]] = deque()
        inflight: Deque[Tuple[int, Future]] = deque()

        def keep_in_flight(n: int) -> None:  # queue whole windows until n pack fetches are running
            while len(inflight) < n:
                item = next(plan)
                queued.append(item)
                inflight.extend((p, pool.submit(self._fetch, p)) for p in item[2])

        try:
            while True:
                keep_in_flight(1)
                epoch, number, window, skip = queued.popleft()
                keep_in_flight(len(window) + self.prefetch)
                loaded: Dict[int, bytes] = {}
                for _ in window:
                    p, fut = inflight.popleft()
                    began = time.perf_counter()
                    loaded[p] = fut.result()
                    self.stats["wait_seconds"] += time.perf_counter() - began
                keep_in_flight(self.prefetch)
                for name in self._shuffled(epoch, number, window)[skip:]:
                    yield self._materialize(name, loaded)
        finally:
            for _, fut in inflight:
                fut.cancel()
            pool.shutdown(wait=True, cancel_futures=True)
