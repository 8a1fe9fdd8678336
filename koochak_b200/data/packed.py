"""Stream the groups of a packed collection to data-loading workers.

(reference: koochak/data/packed.py:77-412)

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
import random
import threading
import time
from collections import OrderedDict, deque
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Callable, Deque, Dict, Iterator, List, Mapping, Optional, Sequence, Tuple

from ..storage.collection import Collection, FileEntry, load_collection, object_key, pack_ranges, read_pack_ranges
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


class PackedGroups:
    def __init__(self, collection: Collection) -> None:
        if not isinstance(collection, Collection):
            raise TypeError("PackedGroups needs a Collection")
        if collection.layout != "packed":
            raise ValueError("PackedGroups needs a collection with the 'packed' layout")
        self.collection = collection
        by_group: Dict[str, List[FileEntry]] = {}
        for e in collection.files:
            by_group.setdefault(e.group, []).append(e)
        groups: Dict[str, GroupInfo] = {}
        first_in: Dict[int, List[str]] = {}
        for name, es in by_group.items():
            es.sort(key=lambda x: (x.pack is None, x.pack or 0, x.offset or 0, x.path))
            groups[name] = GroupInfo(name, tuple(es), es[0].pack, sum(x.size for x in es))
            if es[0].pack is not None:
                first_in.setdefault(es[0].pack, []).append(name)
        loose = sorted(n for n, g in groups.items() if g.pack is None)
        if loose:
            raise ValueError(f"{len(loose)} groups have no packed file (e.g. {loose[:3]}); archive with "
                             "--object-bytes at least as large as --pack-bytes")
        self.groups: Mapping[str, GroupInfo] = MappingProxyType(groups)
        self.pack_groups: Mapping[int, Tuple[str, ...]] = MappingProxyType({
            p: tuple(sorted(ns, key=lambda n: groups[n].files[0].offset or 0)) for p, ns in first_in.items()})

    @classmethod
    def load(cls, store: Store) -> "PackedGroups":
        return cls(load_collection(store))

    def load_group(self, store: Store, name: str, *, verify: bool = True) -> LoadedGroup:
        """One range request per pack the group touches (usually one)."""

        info = self.groups[name]
        per_pack: Dict[int, List[FileEntry]] = {}
        for e in info.files:
            if e.pack is not None:
                per_pack.setdefault(e.pack, []).append(e)
        files: Dict[str, bytes] = {}
        for p, es in per_pack.items():
            lo = min(e.offset for e in es)
            hi = max(e.offset + e.size for e in es)
            span = store.get(self.collection.packs[p].key, lo, hi - lo)
            for e in es:
                files[e.path] = span[e.offset - lo:e.offset - lo + e.size]
        for e in info.files:
            if e.pack is None:
                files[e.path] = store.get(object_key(e.path))
            _check(files[e.path], e, verify)
        return LoadedGroup(name, MappingProxyType(files), MappingProxyType({e.path: e for e in info.files}))

    def read_files(self, store: Store, entries: Sequence[FileEntry], *, verify: bool = True, streams: int = 16,
                   merge_gap: int = 64 * 1024, max_range: int = 16 << 20) -> Dict[str, bytes]:
        uniq = {e.path: e for e in entries}
        per_key: Dict[str, list] = {}
        for part in pack_ranges([e for e in uniq.values() if e.pack is not None], self.collection.packs,
                                merge_gap=merge_gap, max_range=max_range):
            per_key.setdefault(part.pack.key, []).append(part)
        jobs: List[Callable[[], Dict[str, bytes]]] = [
            (lambda parts=parts: read_pack_ranges(store, parts, verify=verify)) for parts in per_key.values()]
        jobs += [(lambda e=e: {e.path: _check(store.get(e.object), e, verify)}) for e in uniq.values()
                 if e.pack is None]
        out: Dict[str, bytes] = {}
        if len(jobs) <= 1 or streams <= 1:
            for j in jobs:
                out.update(j())
            return out
        with ThreadPoolExecutor(max_workers=min(streams, len(jobs))) as pool:
            for part in pool.map(lambda j: j(), jobs):
                out.update(part)
        return out

    def plan(self, *, num_owners: int, seed: int = 0,
             select: Optional[Callable[[str], bool]] = None) -> Tuple[Tuple[int, ...], ...]:
        shards = []
        for p, names in sorted(self.pack_groups.items()):
            n = sum(1 for g in names if select is None or select(g))
            if n:
                pe = self.collection.packs[p]
                shards.append(Shard(pe.key, pe.size, pe.sha256, n))
        if not shards:
            raise ValueError("no pack holds a selected group")
        number = {pe.key: i for i, pe in enumerate(self.collection.packs)}
        owners = plan_shards(shards, num_workers=num_owners, seed=seed)
        return tuple(tuple(sorted(number[s.key] for s in owned)) for owned in owners)


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
            d = self._packs.get(pack)
            if d is not None:
                self._packs.move_to_end(pack)
                self.hits += 1
            return d

    def put(self, pack: int, data: bytes) -> None:
        with self._lock:
            if len(data) > self.max_bytes or pack in self._packs:
                return
            self._packs[pack] = data
            self._bytes += len(data)
            while self._bytes > self.max_bytes:
                _, old = self._packs.popitem(last=False)
                self._bytes -= len(old)


class GroupStream:
    def __init__(self, store: Store, groups: PackedGroups, packs: Sequence[int], *,
                 select: Optional[Callable[[str], bool]] = None, seed: int = 0, window: int = 2, prefetch: int = 2,
                 start: int = 0, verify: bool = True, cache: Optional[PackCache] = None, retries: int = 0,
                 retry_seconds: float = 5.0) -> None:
        for what, v, lo in (("window", window, 1), ("prefetch", prefetch, 0), ("start", start, 0),
                            ("retries", retries, 0)):
            if type(v) is not int or v < lo:
                raise ValueError(f"{what} must be an integer >= {lo}")
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

    def _fetch(self, p: int) -> bytes:
        if self.cache is not None:
            hit = self.cache.get(p)
            if hit is not None:
                self.stats["cache_hits"] += 1
                return hit
        pe = self.groups.collection.packs[p]
        tries = 0
        while True:
            t0 = time.perf_counter()
            try:
                data = self.store.get(pe.key)
                break
            except OSError:
                if tries >= self.retries:
                    raise
                tries += 1
                self.stats["retries"] += 1
                time.sleep(self.retry_seconds)
        self.stats["fetch_seconds"] += time.perf_counter() - t0
        if len(data) != pe.size or (self.verify and hashlib.sha256(data).hexdigest() != pe.sha256):
            raise ValueError(f"{pe.key} does not match its manifest size and SHA256")
        self.stats["packs_fetched"] += 1
        self.stats["bytes_fetched"] += len(data)
        if self.cache is not None:
            self.cache.put(p, data)
        return data

    def _materialize(self, name: str, loaded: Mapping[int, bytes]) -> LoadedGroup:
        info = self.groups.groups[name]
        files: Dict[str, bytes] = {}
        for e in info.files:
            if e.pack in loaded:
                files[e.path] = loaded[e.pack][e.offset:e.offset + e.size]  # the pack was verified whole
                continue
            if e.pack is not None:
                data = self.store.get(self.groups.collection.packs[e.pack].key, e.offset, e.size)
            else:
                data = self.store.get(object_key(e.path))
            files[e.path] = _check(data, e, self.verify)
        return LoadedGroup(name, MappingProxyType(files), MappingProxyType({e.path: e for e in info.files}))

    def _windows(self, epoch: int) -> List[Tuple[int, ...]]:
        keys = self.groups.collection.packs
        order = sorted(self.packs, key=lambda p: _hash_order(self.seed, epoch, keys[p].key))
        return [tuple(order[i:i + self.window]) for i in range(0, len(order), self.window)]

    def _shuffled(self, epoch: int, number: int, window: Sequence[int]) -> List[str]:
        names = [g for p in window for g in self.selected[p]]
        random.Random(_hash_order(self.seed, epoch, f"window-{number}")).shuffle(names)
        return names

    def _schedule(self) -> Iterator[Tuple[int, int, Tuple[int, ...], int]]:
        skip, epoch = self.start, 0
        while True:
            for number, window in enumerate(self._windows(epoch)):
                n = sum(len(self.selected[p]) for p in window)
                if skip >= n:
                    skip -= n
                    continue
                yield epoch, number, window, skip
                skip = 0
            epoch += 1

    def __iter__(self) -> Iterator[LoadedGroup]:
        sched = self._schedule()
        pool = ThreadPoolExecutor(max_workers=max(1, self.prefetch))
        pending: Deque[Tuple[int, int, Tuple[int, ...], int]] = deque()
        fetching: Deque[Tuple[int, Future]] = deque()

        def fill(n: int) -> None:  # schedule whole windows until n fetches are in flight
            while len(fetching) < n:
                item = next(sched)
                pending.append(item)
                fetching.extend((p, pool.submit(self._fetch, p)) for p in item[2])

        try:
            while True:
                fill(1)
                epoch, number, window, skip = pending.popleft()
                fill(len(window) + self.prefetch)
                loaded = {}
                for _ in window:
                    p, fut = fetching.popleft()
                    t0 = time.perf_counter()
                    loaded[p] = fut.result()
                    self.stats["wait_seconds"] += time.perf_counter() - t0
                fill(self.prefetch)
                for name in self._shuffled(epoch, number, window)[skip:]:
                    yield self._materialize(name, loaded)
        finally:
            for _, fut in fetching:
                fut.cancel()
            pool.shutdown(wait=True, cancel_futures=True)
