"""Collections: many files described by one manifest written last.

(behaviour of reference koochak/storage/collection.py:205-411)

Under one store prefix::

    manifest.json               commit point: layout, packs, totals, file-table digest
    files.jsonl.gz              one row per file: path, size, sha256, mode, mtime_ns,
                                group, and either (pack, offset) or object
    packs/pack-000000.tar       plain tar packs of small files (layout "packed")
    objects/<path>              files kept as standalone objects

Readers never list storage: the file table answers listing, ``stat`` and the
location of every byte. A packed file is ``size`` bytes at ``offset`` in its
pack (an ordinary tar member); files of one group are contiguous in a pack so
a group loads with one range read. Tables are deterministic (sorted rows,
canonical JSON, gzip mtime 0), so re-committing the same collection is
accepted and a different one refused. The layout (kind ``koochak.collection``,
version 1) is kept identical to the reference's so either framework reads
collections written by the other.
"""

from __future__ import annotations

import gzip
import hashlib
import json
import re
import tarfile
from dataclasses import dataclass
from fnmatch import fnmatchcase
from types import MappingProxyType
from typing import Any, Dict, Iterable, Iterator, List, Mapping, Optional, Sequence, Tuple

from .store import Store, transient_read_error, validate_key

__all__ = ["COLLECTION_KIND", "FILES_KEY", "LAYOUTS", "MANIFEST_KEY", "Collection", "FileEntry", "PackEntry",
           "PackRange", "load_collection", "member_header", "object_key", "pack_key", "pack_ranges", "put_once",
           "read_pack_range", "read_pack_ranges", "tar_padding", "write_collection", "TAR_END"]

COLLECTION_KIND = "koochak.collection"
VERSION = 1
MANIFEST_KEY = "manifest.json"
FILES_KEY = "files.jsonl.gz"
LAYOUTS = ("packed", "objects")
TAR_BLOCK = 512
TAR_END = b"\0" * (2 * TAR_BLOCK)
_HEX64 = re.compile(r"[0-9a-f]{64}")


def pack_key(index: int) -> str:
    return f"packs/pack-{index:06d}.tar"


def object_key(path: str) -> str:
    return f"objects/{path}"


def tar_padding(size: int) -> bytes:
    return b"\0" * (-size % TAR_BLOCK)


def member_header(path: str, size: int, mode: int, mtime_ns: int) -> bytes:
    """A deterministic tar header for one regular file (PAX for long or non-ASCII names)."""

    ti = tarfile.TarInfo(path)
    ti.size, ti.mode, ti.mtime = size, mode & 0o7777, mtime_ns // 1_000_000_000
    ti.uid = ti.gid = 0
    ti.uname = ti.gname = ""
    ti.type = tarfile.REGTYPE
    return ti.tobuf(format=tarfile.PAX_FORMAT, encoding="utf-8", errors="strict")


def _nonneg(v: object, what: str, lo: int = 0) -> int:
    if type(v) is not int or v < lo:
        raise ValueError(f"{what} must be an integer >= {lo}, got {v!r}")
    return v


def _hex(v: object, what: str) -> str:
    if not isinstance(v, str) or not _HEX64.fullmatch(v):
        raise ValueError(f"{what} must be 64 lowercase hex characters")
    return v


@dataclass(frozen=True)
class FileEntry:
    path: str
    size: int
    sha256: str
    mode: int
    mtime_ns: int
    group: str
    pack: Optional[int] = None
    offset: Optional[int] = None
    object: Optional[str] = None

    def __post_init__(self) -> None:
        validate_key(self.path, "file path")
        _nonneg(self.size, "size")
        _hex(self.sha256, "sha256")
        _nonneg(self.mode, "mode")
        _nonneg(self.mtime_ns, "mtime_ns")
        if not isinstance(self.group, str) or not self.group:
            raise ValueError(f"group of {self.path} must be a non-empty string")
        packed = self.pack is not None or self.offset is not None
        if packed == (self.object is not None):
            raise ValueError(f"{self.path} must live in exactly one of a pack or an object")
        if packed:
            _nonneg(self.pack, "pack")
            _nonneg(self.offset, "offset")
        else:
            validate_key(self.object, "object key")

    def to_row(self) -> Dict[str, Any]:
        row: Dict[str, Any] = {"path": self.path, "size": self.size, "sha256": self.sha256, "mode": self.mode,
                               "mtime_ns": self.mtime_ns, "group": self.group}
        if self.object is not None:
            row["object"] = self.object
        else:
            row.update(pack=self.pack, offset=self.offset)
        return row

    @classmethod
    def from_row(cls, row: object) -> "FileEntry":
        base = {"path", "size", "sha256", "mode", "mtime_ns", "group"}
        if not isinstance(row, dict) or set(row) not in (base | {"object"}, base | {"pack", "offset"}):
            raise ValueError(f"invalid file-table row: {row!r}")
        return cls(**row)


@dataclass(frozen=True)
class PackEntry:
    key: str
    size: int
    sha256: str
    files: int

    def __post_init__(self) -> None:
        validate_key(self.key, "pack key")
        _nonneg(self.size, "pack size")
        _hex(self.sha256, "pack sha256")
        _nonneg(self.files, "pack file count", 1)


@dataclass(frozen=True)
class Collection:
    layout: str
    packs: Tuple[PackEntry, ...]
    files: Tuple[FileEntry, ...]
    metadata: Mapping[str, Any]
    manifest_sha256: str

    @property
    def size_bytes(self) -> int:
        return sum(f.size for f in self.files)

    def select(self, patterns: Sequence[str] = ()) -> Iterator[FileEntry]:
        for f in self.files:
            if not patterns or any(fnmatchcase(f.path, p) for p in patterns):
                yield f


@dataclass(frozen=True)
class PackRange:
    """One read of ``length`` bytes at ``start`` in a pack, covering whole member files."""

    pack: PackEntry
    start: int
    length: int
    members: Tuple[FileEntry, ...]


def _coalesce(members: List[FileEntry], merge_gap: int, max_range: int) -> Iterator[List[FileEntry]]:
    """Runs of offset-sorted members that one read can cover (small gaps, bounded length)."""

    run: List[FileEntry] = []
    for f in members:
        if run:
            first, last = run[0], run[-1]
            gap = f.offset - (last.offset + last.size)
            span = f.offset + f.size - first.offset
            if gap > merge_gap or span > max_range:
                yield run
                run = []
        run.append(f)
    if run:
        yield run


def pack_ranges(files: Iterable[FileEntry], packs: Sequence[PackEntry], *, merge_gap: int,
                max_range: int) -> List[PackRange]:
    """Cover the packed files with few reads: neighbours share a read when the gap is small enough."""

    by_pack: Dict[int, List[FileEntry]] = {}
    for f in files:
        if f.pack is None:
            raise ValueError(f"{f.path} is a standalone object, not a pack member")
        by_pack.setdefault(f.pack, []).append(f)
    ranges: List[PackRange] = []
    for index in sorted(by_pack):
        ordered = sorted(by_pack[index], key=lambda e: e.offset)
        for run in _coalesce(ordered, merge_gap, max_range):
            lo, hi = run[0].offset, run[-1].offset + run[-1].size
            ranges.append(PackRange(packs[index], lo, hi - lo, tuple(run)))
    return ranges


def _members_of(part: PackRange, data: bytes, verify: bool) -> Dict[str, bytes]:
    """Cut one range read into its member files (checking each digest when asked)."""

    if len(data) != part.length:
        raise ValueError(f"{part.pack.key} is shorter than its manifest says")
    view = memoryview(data)
    out: Dict[str, bytes] = {}
    for f in part.members:
        at = f.offset - part.start
        blob = bytes(view[at:at + f.size])
        if verify and hashlib.sha256(blob).hexdigest() != f.sha256:
            raise ValueError(f"{f.path} in {part.pack.key} does not match its SHA256")
        out[f.path] = blob
    return out


def read_pack_range(store: Store, part: PackRange, *, verify: bool = True) -> Dict[str, bytes]:
    return _members_of(part, store.get(part.pack.key, part.start, part.length), verify)


def read_pack_ranges(store: Store, parts: Sequence[PackRange], *, verify: bool = True) -> Dict[str, bytes]:
    """Several ranges of one pack through one open handle (on some mounts an open costs more than a read).

    If the mount drops the handle with a transient error, the ranges not yet
    read are fetched with ranged gets instead.
    """

    if len({p.pack.key for p in parts}) != 1:
        raise ValueError("read_pack_ranges reads ranges of exactly one pack")
    got: Dict[str, bytes] = {}
    todo = sorted(parts, key=lambda r: r.start)
    try:
        with store.open(todo[0].pack.key) as fh:
            while todo:
                fh.seek(todo[0].start)
                got.update(_members_of(todo[0], fh.read(todo[0].length), verify))
                todo.pop(0)
    except OSError as err:
        if not transient_read_error(err):
            raise
        for p in todo:
            got.update(read_pack_range(store, p, verify=verify))
    return got


def _canonical(value: Any) -> bytes:
    return (json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=False, allow_nan=False)
            + "\n").encode("utf-8")


def put_once(store: Store, key: str, data: bytes) -> None:
    """Create ``key``; an identical existing object is accepted, a different one refused."""

    try:
        store.put(key, data)
    except FileExistsError as exc:
        if store.get(key) != data:
            raise FileExistsError(f"{key} already exists with different content") from exc


def _check(layout: str, packs: Sequence[PackEntry], files: Sequence[FileEntry]) -> None:
    if layout not in LAYOUTS:
        raise ValueError(f"layout must be one of {LAYOUTS}, got {layout!r}")
    paths = [f.path for f in files]
    if paths != sorted(paths) or len(set(paths)) != len(paths):
        raise ValueError("file table must be sorted by path with unique paths")
    counts = [0] * len(packs)
    for f in files:
        if f.pack is None:
            continue
        if f.pack >= len(packs):
            raise ValueError(f"{f.path} refers to missing pack {f.pack}")
        if f.offset + f.size > packs[f.pack].size:
            raise ValueError(f"{f.path} extends past the end of its pack")
        counts[f.pack] += 1
    for p, n in zip(packs, counts):
        if p.files != n:
            raise ValueError(f"{p.key} lists {p.files} files but the table has {n}")


def _totals(packs: Sequence[PackEntry], files: Sequence[FileEntry]) -> Dict[str, int]:
    return {"files": len(files), "bytes": sum(f.size for f in files), "packs": len(packs),
            "objects": sum(1 for f in files if f.object is not None)}


_MANIFEST_FIELDS = frozenset({"kind", "v", "layout", "files_table", "packs", "totals", "metadata"})


def _table_bytes(files: Sequence[FileEntry]) -> bytes:
    """The gzip file table: canonical JSON rows sorted by path, gzip mtime 0 (deterministic)."""

    return gzip.compress(b"".join(_canonical(f.to_row()) for f in files), compresslevel=6, mtime=0)


def _manifest_doc(layout: str, table: bytes, packs: Sequence[PackEntry], files: Sequence[FileEntry],
                  metadata: Mapping[str, Any]) -> Dict[str, Any]:
    return {
        "kind": COLLECTION_KIND,
        "v": VERSION,
        "layout": layout,
        "files_table": {"key": FILES_KEY, "size": len(table), "sha256": hashlib.sha256(table).hexdigest()},
        "packs": [{"key": p.key, "size": p.size, "sha256": p.sha256, "files": p.files} for p in packs],
        "totals": _totals(packs, files),
        "metadata": dict(metadata),
    }


def write_collection(store: Store, *, layout: str, packs: Sequence[PackEntry], files: Iterable[FileEntry],
                     metadata: Optional[Mapping[str, Any]] = None) -> Collection:
    """Write the file table, then the manifest (the commit point); re-writing identical content is accepted."""

    rows = tuple(sorted(files, key=lambda f: f.path))
    pack_list = tuple(packs)
    extra = dict(metadata or {})
    _check(layout, pack_list, rows)
    table = _table_bytes(rows)
    put_once(store, FILES_KEY, table)
    manifest = _canonical(_manifest_doc(layout, table, pack_list, rows, extra))
    put_once(store, MANIFEST_KEY, manifest)
    return Collection(layout, pack_list, rows, MappingProxyType(extra), hashlib.sha256(manifest).hexdigest())


def _parse_manifest(raw: bytes) -> Dict[str, Any]:
    try:
        doc = json.loads(raw)
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise ValueError("collection manifest is not valid JSON") from exc
    if not isinstance(doc, dict) or set(doc) != _MANIFEST_FIELDS:
        raise ValueError(f"collection manifest must contain exactly {sorted(_MANIFEST_FIELDS)}")
    if (doc["kind"], doc["v"]) != (COLLECTION_KIND, VERSION):
        raise ValueError("unsupported collection kind or version")
    ref = doc["files_table"]
    if not isinstance(ref, dict) or set(ref) != {"key", "size", "sha256"}:
        raise ValueError("invalid files_table reference")
    if not isinstance(doc["packs"], list) or not all(isinstance(p, dict) for p in doc["packs"]):
        raise ValueError("manifest packs must be a list of objects")
    if not isinstance(doc["metadata"], dict):
        raise ValueError("manifest metadata must be an object")
    return doc


def load_collection(store: Store) -> Collection:
    """Read and cross-check a collection: manifest, file table digest, pack bounds, totals."""

    raw = store.get(MANIFEST_KEY)
    doc = _parse_manifest(raw)
    ref = doc["files_table"]
    table = store.get(validate_key(ref["key"], "files table key"))
    if (len(table), hashlib.sha256(table).hexdigest()) != (ref["size"], ref["sha256"]):
        raise ValueError("file table does not match the manifest's size and SHA256")
    files = tuple(FileEntry.from_row(json.loads(line)) for line in gzip.decompress(table).splitlines())
    packs = tuple(PackEntry(**p) for p in doc["packs"])
    _check(doc["layout"], packs, files)
    if doc["totals"] != _totals(packs, files):
        raise ValueError("manifest totals do not match the file table")
    return Collection(doc["layout"], packs, files, MappingProxyType(doc["metadata"]), hashlib.sha256(raw).hexdigest())
