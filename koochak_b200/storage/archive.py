"""Archive local trees into collections; pull, verify and list them.

(reference: koochak/storage/archive.py:168-813)

``archive(root, store)`` walks a local directory, packs files smaller than
``object_bytes`` into tar packs of about ``pack_bytes`` and stores larger
files as standalone objects, then commits the collection manifest last
(``koochak_b200.storage.collection``):

* a groups table (CSV ``path,group[,order]``) keeps each group's files
  contiguous in one pack, ordered by ``order`` then group name; files not in
  the table are grouped by directory, after the listed groups;
* the plan depends only on file metadata, so every pack's byte layout is
  known before reading; each pack's record (``<pack>.json`` with the member
  digests) is written right after the pack, so a re-run reuses finished packs
  without re-reading them and refuses packs that differ from the plan;
* a source whose size or mtime changed while being read fails the archive;
  symlinks and special files are refused (exclude them with globs);
* ``delete_sources=True`` removes the local files once the committed
  collection has been verified.

``pull`` restores all files or those matching globs, merging nearby pack
members into range reads, checking every SHA-256, restoring mode and mtime
on local targets and skipping targets that already have the right size.
``verify`` checks sizes, or every byte with ``deep=True``.
"""

from __future__ import annotations

import csv
import hashlib
import json
import os
import stat
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from fnmatch import fnmatchcase
from typing import Dict, List, Mapping, Optional, Sequence, Tuple

from .collection import (TAR_END, Collection, FileEntry, PackEntry, load_collection, member_header, object_key,
                         pack_key, pack_ranges, put_once, read_pack_range, tar_padding, write_collection)
from .store import Store, profile_of, validate_key
from .transfer import TransferItem, copy_objects

__all__ = ["SourceFile", "ArchivePlan", "ArchiveReport", "PullReport", "VerifyReport", "archive", "load_groups",
           "load_file_list", "plan_archive", "pull", "scan_source", "verify"]

DEFAULT_PACK_BYTES = 512 * 1024 * 1024
DEFAULT_OBJECT_BYTES = 64 * 1024 * 1024
_LAST = 1 << 62


@dataclass(frozen=True)
class SourceFile:
    path: str
    size: int
    mode: int
    mtime_ns: int
    group: str
    order: int


@dataclass(frozen=True)
class Member:
    source: SourceFile
    offset: int       # of the file's bytes within the pack
    header: bytes


@dataclass(frozen=True)
class PlannedPack:
    index: int
    members: Tuple[Member, ...]
    size: int

    @property
    def key(self) -> str:
        return pack_key(self.index)


@dataclass(frozen=True)
class ArchivePlan:
    packs: Tuple[PlannedPack, ...]
    objects: Tuple[SourceFile, ...]

    @property
    def files(self) -> int:
        return sum(len(p.members) for p in self.packs) + len(self.objects)

    @property
    def stored_bytes(self) -> int:
        return sum(p.size for p in self.packs) + sum(o.size for o in self.objects)


@dataclass(frozen=True)
class ArchiveReport:
    collection: Collection
    packs_written: int
    packs_reused: int
    objects_copied: int
    bytes_read: int
    seconds: float
    deleted_files: int = 0


@dataclass(frozen=True)
class PullReport:
    files: int
    skipped: int
    bytes: int
    seconds: float


@dataclass
class VerifyReport:
    files: int
    bytes: int
    problems: List[str] = field(default_factory=list)

    @property
    def ok(self) -> bool:
        return not self.problems


def load_groups(path) -> Dict[str, Tuple[str, int]]:
    """CSV rows ``path,group[,order]`` (header optional) -> {path: (group, order)}."""

    out: Dict[str, Tuple[str, int]] = {}
    with open(path, newline="", encoding="utf-8") as fh:
        for i, row in enumerate(csv.reader(fh)):
            if not row or (i == 0 and row[0] == "path"):
                continue
            if len(row) not in (2, 3) or not row[1]:
                raise ValueError(f"groups row {i + 1} must be path,group[,order]: {row!r}")
            rel = validate_key(row[0], "groups path")
            if rel in out:
                raise ValueError(f"groups table lists {rel} twice")
            out[rel] = (row[1], int(row[2]) if len(row) == 3 and row[2] != "" else 0)
    return out


def load_file_list(path) -> List[str]:
    with open(path, encoding="utf-8") as fh:
        return [validate_key(line.strip(), "file list entry") for line in fh if line.strip()]


def scan_source(root: str, *, exclude: Sequence[str] = (), include: Optional[Sequence[str]] = None,
                groups: Optional[Mapping[str, Tuple[str, int]]] = None, files: Optional[Sequence[str]] = None,
                skip_symlinks: bool = False, min_age_seconds: float = 0.0) -> List[SourceFile]:
    """Regular files under ``root``: ``exclude`` globs prune, ``include`` globs keep, ``files`` lists exactly."""

    root = os.path.abspath(root)
    wanted = set(files) if files is not None else None
    globs = list(include or [])
    newest = time.time() - float(min_age_seconds)
    out: List[SourceFile] = []
    for d, dirs, names in os.walk(root, followlinks=False):
        dirs.sort()
        for name in sorted(dirs + names):
            full = os.path.join(d, name)
            rel = os.path.relpath(full, root).replace(os.sep, "/")
            if any(fnmatchcase(rel, g) for g in exclude):
                if name in dirs:
                    dirs.remove(name)
                continue
            st = os.lstat(full)
            if stat.S_ISDIR(st.st_mode):
                continue
            if not stat.S_ISREG(st.st_mode):
                if skip_symlinks and stat.S_ISLNK(st.st_mode):
                    continue
                raise ValueError(f"refusing non-regular file (symlink or special): {rel}; exclude it with a glob")
            if wanted is not None and rel not in wanted:
                continue
            if globs and not any(fnmatchcase(rel, g) for g in globs):
                continue
            if min_age_seconds and st.st_mtime > newest:
                continue
            grp, order = (groups or {}).get(rel, (os.path.dirname(rel) or ".", _LAST))
            out.append(SourceFile(validate_key(rel, "path"), st.st_size, stat.S_IMODE(st.st_mode), st.st_mtime_ns,
                                  grp, order))
    return out


def plan_archive(files: Sequence[SourceFile], *, pack_bytes: int = DEFAULT_PACK_BYTES,
                 object_bytes: int = DEFAULT_OBJECT_BYTES) -> ArchivePlan:
    """Lay out every pack (member offsets included) from metadata alone."""

    small = sorted((f for f in files if f.size < object_bytes), key=lambda f: (f.order, f.group, f.path))
    objects = tuple(sorted((f for f in files if f.size >= object_bytes), key=lambda f: f.path))
    packs: List[PlannedPack] = []
    members: List[Member] = []
    size = 0

    def close() -> None:
        nonlocal members, size
        if members:
            packs.append(PlannedPack(len(packs), tuple(members), size + len(TAR_END)))
            members, size = [], 0

    for f in small:
        hdr = member_header(f.path, f.size, f.mode, f.mtime_ns)
        need = len(hdr) + f.size + len(tar_padding(f.size))
        if members and size + need + len(TAR_END) > pack_bytes:
            close()
        members.append(Member(f, size + len(hdr), hdr))
        size += need
    close()
    return ArchivePlan(tuple(packs), objects)


def _read_checked(root: str, f: SourceFile) -> bytes:
    path = os.path.join(root, f.path)
    with open(path, "rb") as fh:
        data = fh.read()
        st = os.fstat(fh.fileno())
    if len(data) != f.size or st.st_size != f.size or st.st_mtime_ns != f.mtime_ns:
        raise ValueError(f"source changed while archiving: {f.path}")
    return data


def _pack_record(pack: PlannedPack, sha: str, digests: Sequence[str]) -> bytes:
    doc = {"key": pack.key, "size": pack.size, "sha256": sha,
           "members": [{"path": m.source.path, "offset": m.offset, "size": m.source.size, "sha256": d}
                       for m, d in zip(pack.members, digests)]}
    return (json.dumps(doc, sort_keys=True, separators=(",", ":")) + "\n").encode()


def _entries(pack: PlannedPack, digests: Sequence[str]) -> List[FileEntry]:
    return [FileEntry(m.source.path, m.source.size, d, m.source.mode, m.source.mtime_ns, m.source.group,
                      pack=pack.index, offset=m.offset) for m, d in zip(pack.members, digests)]


def _reuse(store: Store, pack: PlannedPack) -> Optional[Tuple[PackEntry, List[FileEntry]]]:
    info = store.stat(pack.key)
    if info is None:
        return None
    if info.size != pack.size:
        raise FileExistsError(f"{pack.key} exists with {info.size} bytes but the plan needs {pack.size}")
    rec_key = pack.key + ".json"
    if store.stat(rec_key) is not None:
        rec = json.loads(store.get(rec_key))
    else:  # the pack landed but its record did not: rebuild the record from the stored bytes
        data = store.get(pack.key)
        digests = [hashlib.sha256(data[m.offset:m.offset + m.source.size]).hexdigest() for m in pack.members]
        put_once(store, rec_key, _pack_record(pack, hashlib.sha256(data).hexdigest(), digests))
        rec = json.loads(store.get(rec_key))
    want = [(m.source.path, m.offset, m.source.size) for m in pack.members]
    have = [(r["path"], r["offset"], r["size"]) for r in rec["members"]]
    if have != want:
        raise FileExistsError(f"{pack.key} differs from the archive plan; use a new prefix")
    digests = [r["sha256"] for r in rec["members"]]
    return PackEntry(pack.key, pack.size, rec["sha256"], len(pack.members)), _entries(pack, digests)


def _write_pack(root: str, store: Store, pack: PlannedPack) -> Tuple[PackEntry, List[FileEntry], int]:
    parts: List[bytes] = []
    digests: List[str] = []
    h = hashlib.sha256()
    for m in pack.members:
        data = _read_checked(root, m.source)
        digests.append(hashlib.sha256(data).hexdigest())
        for piece in (m.header, data, tar_padding(m.source.size)):
            parts.append(piece)
            h.update(piece)
    parts.append(TAR_END)
    h.update(TAR_END)
    store.put(pack.key, parts)
    put_once(store, pack.key + ".json", _pack_record(pack, h.hexdigest(), digests))
    return PackEntry(pack.key, pack.size, h.hexdigest(), len(pack.members)), _entries(pack, digests), pack.size


def archive(root: str, store: Store, *, exclude: Sequence[str] = (), groups=None,
            include: Optional[Sequence[str]] = None, pack_bytes: int = DEFAULT_PACK_BYTES,
            object_bytes: Optional[int] = DEFAULT_OBJECT_BYTES, metadata: Optional[Mapping] = None,
            streams: Optional[int] = None, delete_sources: bool = False, layout: str = "packed",
            files: Optional[Sequence[str]] = None, skip_symlinks: bool = False, min_age_seconds: float = 0.0,
            dry_run: bool = False):
    """Archive ``root`` into ``store``; with ``dry_run`` return the ``ArchivePlan`` and write nothing."""

    t0 = time.perf_counter()
    root = os.path.abspath(root)
    if layout not in ("packed", "objects"):
        raise ValueError("layout must be 'packed' or 'objects'")
    table = load_groups(groups) if isinstance(groups, (str, os.PathLike)) else groups
    found = scan_source(root, exclude=exclude, include=include, groups=table, files=files,
                        skip_symlinks=skip_symlinks, min_age_seconds=min_age_seconds)
    if not found:
        raise ValueError(f"nothing to archive under {root}")
    if object_bytes is None:
        object_bytes = max(1, min(DEFAULT_OBJECT_BYTES, pack_bytes))
    plan = plan_archive(found, pack_bytes=pack_bytes, object_bytes=0 if layout == "objects" else object_bytes)
    if dry_run:
        return plan
    workers = streams or profile_of(store).streams
    packs: List[Optional[PackEntry]] = [None] * len(plan.packs)
    entries: List[FileEntry] = []
    written = reused = 0
    nbytes = 0

    def one(p: PlannedPack):
        got = _reuse(store, p)
        if got is not None:
            return p.index, got[0], got[1], 0, True
        pe, fe, n = _write_pack(root, store, p)
        return p.index, pe, fe, n, False

    with ThreadPoolExecutor(max_workers=max(1, workers)) as pool:
        for idx, pe, fe, n, was_reused in pool.map(one, plan.packs):
            packs[idx] = pe
            entries.extend(fe)
            nbytes += n
            reused += was_reused
            written += not was_reused
    objects = 0
    for f in plan.objects:
        key = object_key(f.path)
        data = _read_checked(root, f)
        digest = hashlib.sha256(data).hexdigest()
        info = store.stat(key)
        if info is None:
            store.put(key, data)
            objects += 1
        elif info.size != f.size or hashlib.sha256(store.get(key)).hexdigest() != digest:
            raise FileExistsError(f"{key} exists with different content")
        nbytes += f.size
        entries.append(FileEntry(f.path, f.size, digest, f.mode, f.mtime_ns, f.group, object=key))
    col = write_collection(store, layout="packed" if plan.packs else "objects", packs=[p for p in packs if p],
                           files=entries, metadata=metadata)
    deleted = 0
    if delete_sources:
        rep = verify(store, deep=True)
        if not rep.ok:
            raise ValueError("archive verification failed; sources kept: " + "; ".join(rep.problems[:5]))
        for e in col.files:
            os.unlink(os.path.join(root, e.path))
            deleted += 1
    return ArchiveReport(col, written, reused, objects, nbytes, time.perf_counter() - t0, deleted)


def _restore(path: str, e: FileEntry) -> None:
    os.chmod(path, e.mode)
    os.utime(path, ns=(e.mtime_ns, e.mtime_ns))


def pull(store: Store, target: Store, *, patterns: Sequence[str] = (), merge_gap: int = 1 << 20,
         max_range: int = 64 << 20, streams: Optional[int] = None) -> PullReport:
    """Restore files (all, or those matching ``patterns``) into ``target``; re-runs resume."""

    t0 = time.perf_counter()
    col = load_collection(store)
    want = list(col.select(patterns))
    todo, skipped = [], 0
    for e in want:
        info = target.stat(e.path)
        if info is not None:
            if info.size != e.size:
                raise FileExistsError(f"target {e.path} exists with {info.size} bytes, expected {e.size}")
            skipped += 1
        else:
            todo.append(e)
    packed = [e for e in todo if e.pack is not None]
    nbytes = 0
    workers = streams or profile_of(store).streams

    def fetch(part):
        blobs = read_pack_range(store, part, verify=True)
        n = 0
        for m in part.members:
            target.put(m.path, blobs[m.path])
            n += m.size
            lp = target.local_path(m.path)
            if lp:
                _restore(lp, m)
        return n

    with ThreadPoolExecutor(max_workers=max(1, workers)) as pool:
        for n in pool.map(fetch, pack_ranges(packed, col.packs, merge_gap=merge_gap, max_range=max_range)):
            nbytes += n
    objs = [e for e in todo if e.object is not None]
    if objs:
        rep = copy_objects(store, target, [TransferItem(e.object, e.path, e.size, e.sha256) for e in objs],
                           streams=workers)
        nbytes += rep.bytes_copied
        for e in objs:
            lp = target.local_path(e.path)
            if lp:
                _restore(lp, e)
    return PullReport(len(todo), skipped, nbytes, time.perf_counter() - t0)


def verify(store: Store, *, deep: bool = False, streams: Optional[int] = None) -> VerifyReport:
    col = load_collection(store)
    problems: List[str] = []
    members: Dict[int, List[FileEntry]] = {}
    for e in col.files:
        if e.pack is not None:
            members.setdefault(e.pack, []).append(e)

    def check_pack(i_p):
        i, p = i_p
        out = []
        info = store.stat(p.key)
        if info is None or info.size != p.size:
            return [f"{p.key}: missing or wrong size"]
        if deep:
            data = store.get(p.key)
            if hashlib.sha256(data).hexdigest() != p.sha256:
                out.append(f"{p.key}: SHA256 differs")
            for e in members.get(i, []):
                if hashlib.sha256(data[e.offset:e.offset + e.size]).hexdigest() != e.sha256:
                    out.append(f"{e.path}: SHA256 differs")
        return out

    def check_obj(e):
        info = store.stat(e.object)
        if info is None or info.size != e.size:
            return [f"{e.object}: missing or wrong size"]
        if deep and hashlib.sha256(store.get(e.object)).hexdigest() != e.sha256:
            return [f"{e.object}: SHA256 differs"]
        return []

    with ThreadPoolExecutor(max_workers=max(1, streams or profile_of(store).streams)) as pool:
        for res in pool.map(check_pack, enumerate(col.packs)):
            problems.extend(res)
        for res in pool.map(check_obj, [e for e in col.files if e.object is not None]):
            problems.extend(res)
    return VerifyReport(len(col.files), col.size_bytes, problems)
