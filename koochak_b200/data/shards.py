"""Write-once dataset shards, their index, and the dealing of shards to workers.

(behaviour of reference koochak/data/shards.py:134-569)

A dataset is a set of large immutable shard objects plus one small index
written last. The index (``kind: koochak.shard_index``, ``v: 1``) lists every
shard's key (relative to the index's directory), size, SHA-256 and record
count, plus totals and free-form metadata, as canonical JSON; its own SHA-256
names the dataset version. Training never lists storage and can verify every
byte it reads. The index layout, the tar sample encoding (WebDataset layout:
``key.ext`` members, no timestamps or owners, so equal samples give equal
bytes) and the dealing rule below are kept identical to the reference so
datasets built by either framework load in the other.

``plan_shards`` deals whole shards before anything is read: order the shards
by ``sha256(f"{seed}\\0{epoch}\\0{key}")`` (or keep index order), then give
each shard to the worker whose slice of the record range contains the
shard's record midpoint. It is a pure function of its arguments, so every
rank and DataLoader worker computes the same plan without talking.
"""

from __future__ import annotations

import hashlib
import io
import itertools
import json
import posixpath
import re
import tarfile
from dataclasses import dataclass
from types import MappingProxyType
from typing import Any, Callable, Dict, Iterator, List, Mapping, Optional, Sequence, Tuple, Union

from ..storage.store import Store, validate_key

__all__ = ["DEFAULT_TARGET_BYTES", "INDEX_KIND", "INDEX_VERSION", "TAR", "Shard", "ShardFormat", "ShardIndex",
           "ShardWriter", "assign_shards", "decode_tar_samples", "describe_shard", "encode_tar_sample", "load_index",
           "plan_shards", "read_shard", "worker_coordinates", "write_index"]

INDEX_KIND = "koochak.shard_index"
INDEX_VERSION = 1
DEFAULT_TARGET_BYTES = 256 * 1024 * 1024
_HEX64 = re.compile(r"[0-9a-f]{64}")
_CHUNK = 8 << 20
_BLOCK = 512


def _int(v: object, what: str, lo: Optional[int] = None) -> int:
    if type(v) is not int or (lo is not None and v < lo):
        raise ValueError(f"{what} must be an integer{'' if lo is None else f' >= {lo}'}, got {v!r}")
    return v


def _leaf(v: object, what: str) -> str:
    validate_key(v, what)
    if "/" in v:  # type: ignore[operator]
        raise ValueError(f"{what} must be a single path segment: {v!r}")
    return v  # type: ignore[return-value]


@dataclass(frozen=True)
class Shard:
    key: str
    size_bytes: int
    sha256: str
    records: int

    def __post_init__(self) -> None:
        validate_key(self.key, "shard key")
        _int(self.size_bytes, "size_bytes", 0)
        if not isinstance(self.sha256, str) or not _HEX64.fullmatch(self.sha256):
            raise ValueError(f"sha256 must be 64 lowercase hex characters: {self.sha256!r}")
        _int(self.records, "records", 1)


@dataclass(frozen=True)
class ShardIndex:
    key: str
    shards: Tuple[Shard, ...]
    metadata: Mapping[str, Any]
    sha256: str

    @property
    def records(self) -> int:
        return sum(s.records for s in self.shards)

    @property
    def size_bytes(self) -> int:
        return sum(s.size_bytes for s in self.shards)


def _check_shards(shards: Sequence[Shard]) -> Tuple[Shard, ...]:
    items = tuple(shards)
    if not items:
        raise ValueError("a dataset needs at least one shard")
    if any(not isinstance(s, Shard) for s in items):
        raise TypeError("expected Shard entries")
    if len({s.key for s in items}) != len(items):
        raise ValueError("shard keys must be unique")
    return items


def _canonical(value: Any) -> bytes:
    return (json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=False, allow_nan=False)
            + "\n").encode("utf-8")


def _encode_index(key: str, shards: Tuple[Shard, ...], metadata: Mapping[str, Any]) -> bytes:
    if not isinstance(metadata, Mapping):
        raise ValueError("metadata must be a mapping")
    base = posixpath.dirname(key)
    entries = []
    for s in shards:
        rel = s.key
        if base:
            if not s.key.startswith(base + "/"):
                raise ValueError(f"shard {s.key!r} must live under the index directory {base!r}")
            rel = s.key[len(base) + 1:]
        entries.append({"key": rel, "size_bytes": s.size_bytes, "sha256": s.sha256, "records": s.records})
    return _canonical({"kind": INDEX_KIND, "v": INDEX_VERSION, "records": sum(s.records for s in shards),
                       "size_bytes": sum(s.size_bytes for s in shards), "shards": entries,
                       "metadata": dict(metadata)})


def _decode_index(key: str, data: bytes) -> ShardIndex:
    try:
        doc = json.loads(data)
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError(f"shard index is not valid JSON: {key}") from exc
    want = {"kind", "v", "records", "size_bytes", "shards", "metadata"}
    if not isinstance(doc, dict) or set(doc) != want:
        raise ValueError(f"shard index must contain exactly {sorted(want)}: {key}")
    if doc["kind"] != INDEX_KIND or doc["v"] != INDEX_VERSION:
        raise ValueError(f"unsupported shard index kind/version in {key}")
    if not isinstance(doc["shards"], list) or not isinstance(doc["metadata"], dict):
        raise ValueError(f"malformed shard index: {key}")
    base = posixpath.dirname(key)
    shards = []
    for e in doc["shards"]:
        if not isinstance(e, dict) or set(e) != {"key", "size_bytes", "sha256", "records"}:
            raise ValueError(f"invalid shard entry in {key}: {e!r}")
        rel = validate_key(e["key"], "shard key")
        shards.append(Shard(posixpath.join(base, rel) if base else rel, e["size_bytes"], e["sha256"], e["records"]))
    items = _check_shards(shards)
    if doc["records"] != sum(s.records for s in items) or doc["size_bytes"] != sum(s.size_bytes for s in items):
        raise ValueError(f"shard index totals do not match its entries: {key}")
    return ShardIndex(key, items, MappingProxyType(doc["metadata"]), hashlib.sha256(data).hexdigest())


def write_index(store: Store, key: str, shards: Sequence[Shard], *,
                metadata: Optional[Mapping[str, Any]] = None) -> ShardIndex:
    """Commit a dataset by writing its index; an identical re-commit is accepted."""

    validate_key(key, "index key")
    data = _encode_index(key, _check_shards(shards), metadata or {})
    try:
        store.put(key, data)
    except FileExistsError as exc:
        if store.get(key) != data:
            raise FileExistsError(f"a different shard index already exists at {key}") from exc
    return _decode_index(key, data)


def load_index(store: Store, key: str) -> ShardIndex:
    return _decode_index(validate_key(key, "index key"), store.get(key))


def _digest_object(store: Store, key: str) -> Tuple[int, str]:
    h, n = hashlib.sha256(), 0
    with store.open(key) as fh:
        while True:
            b = fh.read(_CHUNK)
            if not b:
                break
            h.update(b)
            n += len(b)
    return n, h.hexdigest()


def describe_shard(store: Store, key: str, *, records: int) -> Shard:
    size, digest = _digest_object(store, key)
    return Shard(key, size, digest, records)


def read_shard(store: Store, shard: Shard, *, verify: bool = True) -> bytes:
    data = store.get(shard.key)
    if len(data) != shard.size_bytes:
        raise ValueError(f"shard {shard.key} has {len(data)} bytes, index says {shard.size_bytes}")
    if verify and hashlib.sha256(data).hexdigest() != shard.sha256:
        raise ValueError(f"shard {shard.key} does not match its index SHA256")
    return data


# ----------------------------------------------------------------------------- formats

@dataclass(frozen=True)
class ShardFormat:
    """A shard is ``encode(r1) + encode(r2) + ... + trailer``; ``decode`` yields the records back."""

    suffix: str
    encode: Callable[[Any], bytes]
    decode: Callable[[bytes], Iterator[Any]]
    trailer: bytes = b""

    def __post_init__(self) -> None:
        if self.suffix:
            _leaf("x" + self.suffix, "suffix")
        if not isinstance(self.trailer, bytes):
            raise ValueError("trailer must be bytes")


def encode_tar_sample(sample: Mapping[str, Any]) -> bytes:
    """``{"__key__": k, ext: bytes...}`` as adjacent tar members ``k.ext`` (sorted by ext)."""

    if not isinstance(sample, Mapping) or "__key__" not in sample:
        raise ValueError("a tar sample must be a mapping with a '__key__' entry")
    key = validate_key(sample["__key__"], "sample '__key__'")
    if "." in posixpath.basename(key):
        raise ValueError(f"sample '__key__' basename must not contain '.': {key!r}")
    fields = sorted((k, v) for k, v in sample.items() if k != "__key__")
    if not fields:
        raise ValueError(f"sample {key!r} has no fields")
    out = bytearray()
    for name, value in fields:
        if not isinstance(name, str) or not name or "/" in name or "\x00" in name:
            raise ValueError(f"sample field names must be non-empty and contain no '/': {name!r}")
        if not isinstance(value, (bytes, bytearray, memoryview)):
            raise TypeError(f"sample field {name!r} must be bytes, got {type(value).__name__}")
        payload = bytes(value)
        ti = tarfile.TarInfo(f"{key}.{name}")
        ti.size, ti.mtime, ti.mode, ti.uid, ti.gid, ti.uname, ti.gname = len(payload), 0, 0o444, 0, 0, "", ""
        out += ti.tobuf(format=tarfile.PAX_FORMAT, encoding="utf-8", errors="strict")
        out += payload + b"\0" * (-len(payload) % _BLOCK)
    return bytes(out)


def decode_tar_samples(data: bytes) -> Iterator[Dict[str, Any]]:
    with tarfile.open(fileobj=io.BytesIO(data), mode="r:") as tf:
        cur: Optional[Dict[str, Any]] = None
        for m in tf:
            if not m.isreg():
                raise ValueError(f"unsupported tar member (not a regular file): {m.name}")
            d, base = posixpath.split(m.name)
            stem, dot, ext = base.partition(".")
            if not stem or not dot or not ext:
                raise ValueError(f"tar member name must look like 'key.ext': {m.name}")
            key = posixpath.join(d, stem) if d else stem
            if cur is None or cur["__key__"] != key:
                if cur is not None:
                    yield cur
                cur = {"__key__": key}
            if ext in cur:
                raise ValueError(f"duplicate field {ext!r} in sample {key!r}")
            fh = tf.extractfile(m)
            cur[ext] = fh.read() if fh is not None else b""
        if cur is not None:
            yield cur


TAR = ShardFormat(".tar", encode_tar_sample, decode_tar_samples, trailer=b"\0" * (2 * _BLOCK))


# ----------------------------------------------------------------------------- writer

class _OpenShard:
    """The records of the shard being filled: encoded pieces, their running size and digest."""

    def __init__(self) -> None:
        self.pieces: List[bytes] = []
        self.size = 0
        self.count = 0
        self.digest = hashlib.sha256()

    def append(self, encoded: bytes) -> None:
        self.pieces.append(encoded)
        self.digest.update(encoded)
        self.size += len(encoded)
        self.count += 1

    def seal(self, key: str, trailer: bytes) -> Tuple[Shard, List[bytes]]:
        self.digest.update(trailer)
        return Shard(key, self.size + len(trailer), self.digest.hexdigest(), self.count), self.pieces + [trailer]


class ShardWriter:
    """Pack records into ``{prefix}/{name}-{n:06d}{suffix}`` shards of about ``target_bytes``; index last.

    Leaving the ``with`` block by an exception commits nothing. Encoding is
    deterministic, so re-running an interrupted build accepts the identical
    shards it left behind and refuses any that differ.
    """

    def __init__(self, store: Store, prefix: str, *, format: ShardFormat = TAR,
                 target_bytes: int = DEFAULT_TARGET_BYTES, name: str = "shard", index_name: str = "index.json",
                 metadata: Optional[Mapping[str, Any]] = None) -> None:
        if prefix != "":
            validate_key(prefix, "prefix")
        if not isinstance(format, ShardFormat):
            raise TypeError("format must be a ShardFormat")
        self.store, self.prefix, self.format = store, prefix, format
        self.target_bytes = _int(target_bytes, "target_bytes", 1)
        self.name = _leaf(name, "name")
        self.index_name = _leaf(index_name, "index_name")
        self.metadata = dict(metadata or {})
        self.index: Optional[ShardIndex] = None
        self._written: List[Shard] = []
        self._current = _OpenShard()
        self._state = "open"

    def _key(self, leaf: str) -> str:
        return f"{self.prefix}/{leaf}" if self.prefix else leaf

    def _require_open(self) -> None:
        if self._state != "open":
            raise RuntimeError(f"ShardWriter is {self._state}")

    def add(self, record: Any) -> None:
        self._require_open()
        encoded = self.format.encode(record)
        if not isinstance(encoded, bytes):
            raise TypeError(f"format.encode must return bytes, got {type(encoded).__name__}")
        self._current.append(encoded)
        if self._current.size + len(self.format.trailer) >= self.target_bytes:
            self._emit()

    def _emit(self) -> None:
        if self._current.count == 0:
            return
        name = self._key(f"{self.name}-{len(self._written):06d}{self.format.suffix}")
        shard, body = self._current.seal(name, self.format.trailer)
        try:
            self.store.put(shard.key, body)
        except FileExistsError as exc:
            # A rerun of an interrupted build: the same bytes are fine, anything else is not.
            if _digest_object(self.store, shard.key) != (shard.size_bytes, shard.sha256):
                raise FileExistsError(f"{shard.key} already exists with different content; delete the "
                                      "uncommitted shards or choose a new prefix") from exc
        self._written.append(shard)
        self._current = _OpenShard()

    def close(self) -> ShardIndex:
        if self._state == "closed":
            assert self.index is not None
            return self.index
        self._require_open()
        try:
            self._emit()
            if not self._written:
                raise ValueError("no records were added; refusing to commit an empty dataset")
            self.index = write_index(self.store, self._key(self.index_name), self._written, metadata=self.metadata)
        except BaseException:
            self._state = "aborted"
            raise
        self._state = "closed"
        return self.index

    def abort(self) -> None:
        if self._state == "open":
            self._state = "aborted"
            self._current = _OpenShard()

    def __enter__(self) -> "ShardWriter":
        return self

    def __exit__(self, exc_type, exc, tb) -> None:
        self.close() if exc_type is None else self.abort()


# ----------------------------------------------------------------------------- planning

ShardsLike = Union[ShardIndex, Sequence[Shard]]


def _shuffle_rank(seed: int, epoch: int, key: str) -> bytes:
    """Sort key of a shard for one (seed, epoch): a hash, so every process computes the same order."""

    return hashlib.sha256(f"{seed}\x00{epoch}\x00{key}".encode("utf-8")).digest()


def plan_shards(shards: ShardsLike, *, num_workers: int, epoch: int = 0, seed: int = 0,
                shuffle: bool = True) -> Tuple[Tuple[Shard, ...], ...]:
    """Deal whole shards to ``num_workers`` workers (a pure function: every process gets the same plan).

    Shards are ordered by ``_shuffle_rank`` (or kept in index order), laid
    end to end on the record axis, and each goes to the worker whose equal
    slice of that axis contains the shard's midpoint.
    """

    _int(num_workers, "num_workers", 1)
    _int(epoch, "epoch", 0)
    _int(seed, "seed")
    if not isinstance(shuffle, bool):
        raise ValueError("shuffle must be a boolean")
    items = _check_shards(shards.shards if isinstance(shards, ShardIndex) else shards)
    if len(items) < num_workers:
        raise ValueError(f"{len(items)} shards cannot feed {num_workers} workers; write smaller shards or use "
                         "fewer workers")
    ordered = sorted(items, key=lambda sh: _shuffle_rank(seed, epoch, sh.key)) if shuffle else list(items)
    counts = [sh.records for sh in ordered]
    starts = [0, *itertools.accumulate(counts)][:-1]
    total = starts[-1] + counts[-1]
    hands: List[List[Shard]] = [[] for _ in range(num_workers)]
    for shard, start, n in zip(ordered, starts, counts):
        # midpoint start + n/2 scaled to [0, num_workers), in exact integer arithmetic
        hands[(2 * start + n) * num_workers // (2 * total)].append(shard)
    empty = [w for w, hand in enumerate(hands) if not hand]
    if empty:
        raise ValueError(f"shard record counts are too uneven to give all {num_workers} workers a shard "
                         f"(idle workers include {empty[:8]}); write smaller shards or use fewer workers")
    return tuple(tuple(hand) for hand in hands)


def assign_shards(shards: ShardsLike, *, worker: int, num_workers: int, epoch: int = 0, seed: int = 0,
                  shuffle: bool = True) -> Tuple[Shard, ...]:
    _int(num_workers, "num_workers", 1)
    if type(worker) is not int or not 0 <= worker < num_workers:
        raise ValueError(f"worker must be in [0, {num_workers}), got {worker!r}")
    return plan_shards(shards, num_workers=num_workers, epoch=epoch, seed=seed, shuffle=shuffle)[worker]


def worker_coordinates(*, rank: int, world_size: int) -> Tuple[int, int]:
    """(worker, num_workers) over every rank x DataLoader worker; call inside ``__iter__``."""

    _int(world_size, "world_size", 1)
    if type(rank) is not int or not 0 <= rank < world_size:
        raise ValueError(f"rank must be in [0, {world_size}), got {rank!r}")
    import torch.utils.data

    info = torch.utils.data.get_worker_info()
    local, per = (0, 1) if info is None else (info.id, info.num_workers)
    return rank * per + local, world_size * per
