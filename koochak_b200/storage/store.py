"""Write-once object stores (reference: koochak/storage/store.py:76-595).

A store maps relative ``/``-separated keys to immutable objects. ``put`` is
create-only and returns only when the exact bytes are readable, so writing a
small manifest last is a commit point on any backend. There is no rename,
append, overwrite or symlink in the contract.

Locations: plain paths and ``file://`` URIs are :class:`LocalStore`; other
``scheme://`` URIs come from the stores file, :func:`register_store`, or the
``koochak.stores`` entry-point group.
"""

from __future__ import annotations

import errno
import hashlib
import math
import os
import stat
import tempfile
import time
from dataclasses import dataclass
from importlib import metadata
from typing import Any, BinaryIO, Callable, Dict, Iterable, Iterator, List, Optional, Protocol, Union, runtime_checkable
from urllib.parse import unquote, urlparse

import re

from ..utils.paths import canonical_dir
from .atomic import _fsync_directory

__all__ = ["DEFAULT_PROFILE", "ENTRY_POINT_GROUP", "LOCAL_PROFILE", "LocalStore", "ObjectInfo", "Store",
           "StoreProfile", "min_object_bytes", "open_store", "profile_of", "register_store", "validate_key",
           "validate_scheme", "transient_read_error"]

ENTRY_POINT_GROUP = "koochak.stores"
PutData = Union[bytes, bytearray, memoryview, Iterable[Union[bytes, bytearray, memoryview]]]
StoreFactory = Callable[[str], "Store"]

_TEMP_MARKER = ".koochak-put-"
_SCHEME_RX = re.compile(r"[a-z][a-z0-9+.-]*")
_PUBLISH_MODES = ("link", "exclusive")
_CHUNK = 8 << 20
_NO_HARDLINK = frozenset(getattr(errno, n) for n in ("EPERM", "ENOTSUP", "EOPNOTSUPP", "ENOSYS", "EXDEV")
                         if hasattr(errno, n))
# Transient read failures on object-storage mounts: a close still committing on
# another node (ETIME, EIO) or the mount's client briefly losing its service.
_SETTLING = (errno.ETIME, errno.EIO, errno.ECONNABORTED, errno.ECONNRESET, errno.ENOTCONN)


@dataclass(frozen=True, slots=True)
class ObjectInfo:
    key: str
    size: int
    sha256: Optional[str] = None


@dataclass(frozen=True, slots=True)
class StoreProfile:
    """Measured performance of a store; upper layers derive defaults from it."""

    request_seconds: float = 0.001
    stream_mb_s: float = 500.0
    streams: int = 4
    range_streams: int = 1
    part_bytes: int = 64 * 1024 * 1024
    list_is_cheap: bool = True

    def __post_init__(self) -> None:
        for name in ("request_seconds", "stream_mb_s"):
            v = getattr(self, name)
            if isinstance(v, bool) or not isinstance(v, (int, float)):
                raise ValueError(f"{name} must be a number")
            if not math.isfinite(v) or v <= 0:
                raise ValueError(f"{name} must be positive and finite")
        for name in ("streams", "range_streams", "part_bytes"):
            v = getattr(self, name)
            if type(v) is not int or v < 1:
                raise ValueError(f"{name} must be a positive integer")
        if not isinstance(self.list_is_cheap, bool):
            raise ValueError("list_is_cheap must be a boolean")


LOCAL_PROFILE = StoreProfile()
DEFAULT_PROFILE = StoreProfile(request_seconds=0.1, stream_mb_s=50.0, streams=16, range_streams=1,
                               part_bytes=32 * 1024 * 1024, list_is_cheap=False)


def profile_of(store: "Store") -> StoreProfile:
    prof = getattr(store, "profile", None)
    if prof is None:
        return DEFAULT_PROFILE
    if not isinstance(prof, StoreProfile):
        raise TypeError(f"{type(store).__name__}.profile must be a StoreProfile")
    return prof


def min_object_bytes(profile: StoreProfile, *, max_overhead: float = 0.25) -> int:
    """Smallest object whose per-request overhead stays at or below ``max_overhead``."""

    if not 0 < max_overhead < 1:
        raise ValueError("max_overhead must be between 0 and 1")
    return int(profile.request_seconds * profile.stream_mb_s * 1e6 * (1 - max_overhead) / max_overhead)


@runtime_checkable
class Store(Protocol):
    def get(self, key: str, offset: int = 0, length: Optional[int] = None) -> bytes: ...
    def open(self, key: str) -> BinaryIO: ...
    def put(self, key: str, data: PutData) -> ObjectInfo: ...
    def stat(self, key: str) -> Optional[ObjectInfo]: ...
    def list(self, prefix: str = "") -> List[str]: ...
    def delete(self, key: str) -> None: ...
    def local_path(self, key: str) -> Optional[str]: ...


def validate_key(key: object, label: str = "key") -> str:
    if not isinstance(key, str) or not key:
        raise ValueError(f"{label} must be a non-empty string")
    if "\x00" in key or "\\" in key:
        raise ValueError(f"{label} must not contain NUL or backslash: {key!r}")
    for seg in key.split("/"):
        if seg in ("", ".", ".."):
            raise ValueError(f"{label} must be relative, without empty, '.' or '..' segments: {key!r}")
        if _TEMP_MARKER in seg:
            raise ValueError(f"{label} must not contain {_TEMP_MARKER!r}: {key!r}")
    return key


def _validate_prefix(prefix: object) -> str:
    if prefix == "":
        return ""
    if not isinstance(prefix, str):
        raise ValueError("prefix must be a string")
    validate_key(prefix[:-1] if prefix.endswith("/") else prefix, "prefix")
    return prefix


def _check_range(offset: object, length: object) -> None:
    if type(offset) is not int or offset < 0:
        raise ValueError("offset must be a non-negative integer")
    if length is not None and (type(length) is not int or length < 0):
        raise ValueError("length must be a non-negative integer or None")


def _chunks(data: PutData) -> Iterator[Union[bytes, bytearray, memoryview]]:
    if isinstance(data, (bytes, bytearray, memoryview)):
        yield data
        return
    if isinstance(data, str):
        raise TypeError("put data must be bytes or an iterable of bytes, not str")
    for c in data:
        if not isinstance(c, (bytes, bytearray, memoryview)):
            raise TypeError(f"put data chunks must be bytes-like, got {type(c).__name__}")
        yield c


def _digest_file(path: str) -> tuple[int, str]:
    h = hashlib.sha256()
    n = 0
    with open(path, "rb") as fh:
        while True:
            block = fh.read(_CHUNK)
            if not block:
                break
            h.update(block)
            n += len(block)
    return n, h.hexdigest()


def transient_read_error(error: BaseException) -> bool:
    return isinstance(error, OSError) and error.errno in _SETTLING


class LocalStore:
    """Store over a POSIX directory tree.

    ``publish="link"`` writes a hidden temp file and hard-links it into place
    (readers never see a partial object; an existing key is never replaced).
    ``publish="exclusive"`` creates the final name with ``O_EXCL`` for mounts
    with neither rename nor hard links. ``verify_readback`` re-reads new
    objects until size and SHA-256 match (up to ``settle_seconds``);
    ``read_settle_seconds`` retries reads that fail transiently.
    """

    def __init__(self, root: Union[str, "os.PathLike[str]"], *, publish: str = "link", fsync: bool = True,
                 verify_readback: bool = False, settle_seconds: float = 0.0, file_mode: int = 0o444,
                 profile: Optional[StoreProfile] = None, read_settle_seconds: float = 0.0) -> None:
        if publish not in _PUBLISH_MODES:
            raise ValueError(f"publish must be one of {_PUBLISH_MODES}, got {publish!r}")
        if not isinstance(fsync, bool) or not isinstance(verify_readback, bool):
            raise ValueError("fsync and verify_readback must be booleans")
        settle = float(settle_seconds)
        if not math.isfinite(settle) or settle < 0:
            raise ValueError("settle_seconds must be a finite, non-negative number")
        if settle > 0 and not verify_readback:
            raise ValueError("settle_seconds requires verify_readback=True")
        if type(file_mode) is not int or not 0 <= file_mode <= 0o777:
            raise ValueError("file_mode must be a permission mode between 0 and 0o777")
        read_settle = float(read_settle_seconds)
        if not math.isfinite(read_settle) or read_settle < 0:
            raise ValueError("read_settle_seconds must be a finite, non-negative number")
        if profile is not None and not isinstance(profile, StoreProfile):
            raise TypeError("profile must be a StoreProfile")
        self.root = canonical_dir(os.fspath(root))
        self.publish = publish
        self.fsync = fsync
        self.verify_readback = verify_readback
        self.settle_seconds = settle
        self.read_settle_seconds = read_settle
        self.file_mode = file_mode
        self.profile = LOCAL_PROFILE if profile is None else profile

    def __repr__(self) -> str:
        return (f"LocalStore({self.root!r}, publish={self.publish!r}, fsync={self.fsync}, "
                f"verify_readback={self.verify_readback}, settle_seconds={self.settle_seconds})")

    def _path(self, key: str) -> str:
        return os.path.join(self.root, *validate_key(key).split("/"))

    def _retrying(self, read: Callable[[], Any]) -> Any:
        deadline = time.monotonic() + self.read_settle_seconds
        while True:
            try:
                return read()
            except OSError as exc:
                if exc.errno not in _SETTLING or time.monotonic() >= deadline:
                    raise
            time.sleep(min(5.0, max(0.0, deadline - time.monotonic())))

    def get(self, key: str, offset: int = 0, length: Optional[int] = None) -> bytes:
        _check_range(offset, length)
        path = self._path(key)

        def read() -> bytes:
            with open(path, "rb") as fh:
                if offset:
                    fh.seek(offset)
                return fh.read() if length is None else fh.read(length)

        return self._retrying(read)

    def open(self, key: str) -> BinaryIO:
        path = self._path(key)
        return self._retrying(lambda: open(path, "rb"))

    def put(self, key: str, data: PutData) -> ObjectInfo:
        path = self._path(key)
        directory = os.path.dirname(path)
        os.makedirs(directory, exist_ok=True)
        size, digest = self._put_link(path, directory, data) if self.publish == "link" else self._put_exclusive(path, data)
        if self.fsync:
            _fsync_directory(directory)
        if self.verify_readback:
            self._await_readback(path, size, digest)
        return ObjectInfo(key, size, digest)

    def _write_all(self, fh: BinaryIO, data: PutData) -> tuple[int, str]:
        h = hashlib.sha256()
        n = 0
        for c in _chunks(data):
            fh.write(c)
            h.update(c)
            n += len(c)
        fh.flush()
        if self.fsync:
            os.fsync(fh.fileno())
        return n, h.hexdigest()

    def _put_link(self, path: str, directory: str, data: PutData) -> tuple[int, str]:
        fd, tmp = tempfile.mkstemp(prefix=f".{os.path.basename(path)}{_TEMP_MARKER}", dir=directory)
        try:
            with os.fdopen(fd, "wb") as fh:
                result = self._write_all(fh, data)
            os.chmod(tmp, self.file_mode)
            try:
                os.link(tmp, path)
            except FileExistsError:
                raise
            except OSError as exc:
                if exc.errno in _NO_HARDLINK:
                    raise OSError(exc.errno, f"{self.root} does not support hard links; use "
                                             "LocalStore(..., publish='exclusive') on this mount") from exc
                raise
            return result
        finally:
            try:
                os.unlink(tmp)
            except FileNotFoundError:
                pass

    def _put_exclusive(self, path: str, data: PutData) -> tuple[int, str]:
        flags = os.O_WRONLY | os.O_CREAT | os.O_EXCL | getattr(os, "O_NOFOLLOW", 0) | getattr(os, "O_CLOEXEC", 0)
        fd = os.open(path, flags, self.file_mode)
        try:
            with os.fdopen(fd, "wb") as fh:
                return self._write_all(fh, data)
        except BaseException:
            try:
                os.unlink(path)  # this call created it, so it owns the partial object
            except FileNotFoundError:
                pass
            raise

    def _await_readback(self, path: str, size: int, digest: str) -> None:
        deadline = time.monotonic() + self.settle_seconds
        last: Optional[OSError] = None
        while True:
            try:
                if _digest_file(path) == (size, digest):
                    return
            except OSError as exc:
                last = exc
            if time.monotonic() >= deadline:
                extra = f" (last error: {last})" if last is not None else ""
                raise OSError(f"{path} did not read back with the written size and SHA256 within "
                              f"{self.settle_seconds}s{extra}")
            time.sleep(min(1.0, max(0.0, deadline - time.monotonic())))

    def stat(self, key: str) -> Optional[ObjectInfo]:
        path = self._path(key)
        try:
            st = self._retrying(lambda: os.stat(path))
        except (FileNotFoundError, NotADirectoryError):
            return None
        return ObjectInfo(key, st.st_size) if stat.S_ISREG(st.st_mode) else None

    def list(self, prefix: str = "") -> List[str]:
        prefix = _validate_prefix(prefix)
        head = prefix.rpartition("/")[0]
        base = os.path.join(self.root, *head.split("/")) if head else self.root
        if not os.path.isdir(base):
            return []
        keys: List[str] = []
        for directory, subdirs, files in os.walk(base):
            rel = os.path.relpath(directory, self.root)
            parent = "" if rel == "." else rel.replace(os.sep, "/") + "/"
            subdirs[:] = [d for d in subdirs
                          if (parent + d).startswith(prefix) or prefix.startswith(parent + d + "/")]
            for f in files:
                if f.startswith(".") and _TEMP_MARKER in f:
                    continue
                key = parent + f
                if key.startswith(prefix):
                    keys.append(key)
        return sorted(keys)

    def delete(self, key: str) -> None:
        try:
            os.remove(self._path(key))
        except FileNotFoundError:
            pass

    def local_path(self, key: str) -> Optional[str]:
        return self._path(key)


_FACTORIES: Dict[str, StoreFactory] = {}


def _uri_subpath(location: str) -> str:
    rest = location.split("://", 1)[1]
    if "?" in rest or "#" in rest:
        raise ValueError(f"store URIs take no query or fragment: {location!r}")
    rest = rest[:-1] if rest.endswith("/") else rest
    return "" if not rest else validate_key(unquote(rest), "store URI path")


def validate_scheme(scheme: object) -> str:
    if not isinstance(scheme, str) or not _SCHEME_RX.fullmatch(scheme):
        raise ValueError(f"invalid store scheme {scheme!r}")
    if scheme == "file":
        raise ValueError("the 'file' scheme is built in")
    return scheme


def register_store(scheme: str, factory: StoreFactory) -> None:
    validate_scheme(scheme)
    if not callable(factory):
        raise TypeError("store factory must be callable")
    prior = _FACTORIES.get(scheme)
    if prior is not None and prior is not factory:
        raise ValueError(f"store scheme {scheme!r} is already registered")
    _FACTORIES[scheme] = factory


def _entry_points():
    return list(metadata.entry_points(group=ENTRY_POINT_GROUP))


def _plugin_provides(scheme: str) -> bool:
    return scheme in _FACTORIES or any(ep.name == scheme for ep in _entry_points())


def _factory(scheme: str, file_schemes: Iterable[str] = ()) -> StoreFactory:
    if scheme in _FACTORIES:
        return _FACTORIES[scheme]
    eps = _entry_points()
    matches = [ep for ep in eps if ep.name == scheme]
    if not matches:
        known = sorted({"file", *_FACTORIES, *(ep.name for ep in eps), *file_schemes})
        raise ValueError(f"no store is registered for scheme {scheme!r}; known schemes: {known}")
    if len(matches) > 1:
        raise ValueError(f"several installed packages provide store scheme {scheme!r}: "
                         f"{sorted(ep.value for ep in matches)}")
    fac = matches[0].load()
    register_store(scheme, fac)
    return fac


def open_store(location: Union[str, "os.PathLike[str]", Store], *,
               stores_file: Optional[Union[str, "os.PathLike[str]"]] = None) -> Store:
    if isinstance(location, Store):
        return location
    text = os.fspath(location)
    if not isinstance(text, str) or not text:
        raise ValueError("store location must be a non-empty string or path")
    if "://" not in text:
        return LocalStore(text)
    parsed = urlparse(text)
    scheme = parsed.scheme.lower()
    if scheme == "file":
        if parsed.netloc not in ("", "localhost") or parsed.params or parsed.query or parsed.fragment:
            raise ValueError(f"file URIs must be file:///absolute/path, got {text!r}")
        return LocalStore(unquote(parsed.path))
    from .stores_file import load_default_or_given

    specs = load_default_or_given(stores_file)
    spec = specs.get(scheme)
    if spec is not None:
        if _plugin_provides(scheme):
            raise ValueError(f"store scheme {scheme!r} is defined by both the stores file and a plugin")
        return spec.open(_uri_subpath(text))
    store = _factory(scheme, specs)(text)
    if not isinstance(store, Store):
        raise TypeError(f"store factory for {scheme!r} returned {type(store).__name__}, which is not a Store")
    return store
