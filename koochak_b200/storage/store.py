"""Write-once object stores.

(behaviour of reference koochak/storage/store.py:76-595)

A store maps relative ``/``-separated keys to immutable objects. ``put`` is
create-only and returns once exactly those bytes are readable, so writing a
small manifest last is a commit point on every backend. There is no rename,
append, overwrite or symlink in the contract.

Where stores come from (``open_store``): a plain path or ``file://`` URI is a
``LocalStore``; any other ``scheme://`` URI is resolved through the
``StoreRegistry`` -- a scheme defined in the private stores file, a factory
registered at run time (``register_store``), or a package's ``koochak.stores``
entry point. A scheme may come from exactly one of these.

``LocalStore`` publishes each object in one of two ways (``publish``):
``"link"`` writes a hidden temporary file and hard-links it to the final
name (readers never see a partial object, an existing key is never
replaced); ``"exclusive"`` creates the final name with ``O_EXCL`` (mounts
without rename or hard links). Mounts over object storage may need a
read-back check after writing (``verify_readback`` / ``settle_seconds``) and
retries of reads that fail while another node's close is still committing
(``read_settle_seconds``).
"""

from __future__ import annotations

import errno
import hashlib
import math
import os
import re
import stat
import tempfile
import time
from dataclasses import dataclass
from importlib import metadata
from typing import Any, BinaryIO, Callable, Dict, Iterable, Iterator, List, Optional, Protocol, Tuple, Union, \
    runtime_checkable
from urllib.parse import unquote, urlparse

from ..utils.paths import canonical_dir
from .atomic import _fsync_directory

__all__ = ["DEFAULT_PROFILE", "ENTRY_POINT_GROUP", "LOCAL_PROFILE", "LocalStore", "ObjectInfo", "Store",
           "StoreProfile", "StoreRegistry", "min_object_bytes", "open_store", "profile_of", "register_store",
           "validate_key", "validate_scheme", "transient_read_error"]

ENTRY_POINT_GROUP = "koochak.stores"
PutData = Union[bytes, bytearray, memoryview, Iterable[Union[bytes, bytearray, memoryview]]]
StoreFactory = Callable[[str], "Store"]

_TEMP_MARKER = ".koochak-put-"  # inside the hidden temporary names of link publication
_BLOCK = 8 << 20
# Link publication falls back to nothing: these mean "this mount has no hard links".
_NO_HARDLINK = {getattr(errno, n) for n in ("EPERM", "ENOTSUP", "EOPNOTSUPP", "ENOSYS", "EXDEV") if hasattr(errno, n)}
# Read errors that pass on object-storage mounts (a close still committing on
# another node, or the mount's client briefly losing its service).
_TRANSIENT = {errno.ETIME, errno.EIO, errno.ECONNABORTED, errno.ECONNRESET, errno.ENOTCONN}


@dataclass(frozen=True, slots=True)
class ObjectInfo:
    key: str
    size: int
    sha256: Optional[str] = None


def _require(ok: bool, message: str, kind=ValueError) -> None:
    if not ok:
        raise kind(message)


@dataclass(frozen=True, slots=True)
class StoreProfile:
    """How a store performs; upper layers size their requests from it."""

    request_seconds: float = 0.001
    stream_mb_s: float = 500.0
    streams: int = 4
    range_streams: int = 1
    part_bytes: int = 64 * 1024 * 1024
    list_is_cheap: bool = True

    def __post_init__(self) -> None:
        for name in ("request_seconds", "stream_mb_s"):
            v = getattr(self, name)
            _require(isinstance(v, (int, float)) and not isinstance(v, bool), f"{name} must be a number")
            _require(math.isfinite(v) and v > 0, f"{name} must be positive and finite")
        for name in ("streams", "range_streams", "part_bytes"):
            v = getattr(self, name)
            _require(type(v) is int and v >= 1, f"{name} must be a positive integer")
        _require(isinstance(self.list_is_cheap, bool), "list_is_cheap must be a boolean")


LOCAL_PROFILE = StoreProfile()
DEFAULT_PROFILE = StoreProfile(request_seconds=0.1, stream_mb_s=50.0, streams=16, range_streams=1,
                               part_bytes=32 * 1024 * 1024, list_is_cheap=False)


def profile_of(store: "Store") -> StoreProfile:
    """The store's declared profile, or the conservative default for stores that declare none."""

    found = getattr(store, "profile", None)
    if found is None:
        return DEFAULT_PROFILE
    _require(isinstance(found, StoreProfile), f"{type(store).__name__}.profile must be a StoreProfile", TypeError)
    return found


def min_object_bytes(profile: StoreProfile, *, max_overhead: float = 0.25) -> int:
    """Smallest object for which the per-request latency costs at most ``max_overhead`` of the transfer."""

    _require(0 < max_overhead < 1, "max_overhead must be between 0 and 1")
    bytes_during_one_request = profile.request_seconds * profile.stream_mb_s * 1e6
    return int(bytes_during_one_request * (1 - max_overhead) / max_overhead)


@runtime_checkable
class Store(Protocol):
    def get(self, key: str, offset: int = 0, length: Optional[int] = None) -> bytes: ...
    def open(self, key: str) -> BinaryIO: ...
    def put(self, key: str, data: PutData) -> ObjectInfo: ...
    def stat(self, key: str) -> Optional[ObjectInfo]: ...
    def list(self, prefix: str = "") -> List[str]: ...
    def delete(self, key: str) -> None: ...
    def local_path(self, key: str) -> Optional[str]: ...


# ----------------------------------------------------------------------------- keys and arguments


def validate_key(key: object, label: str = "key") -> str:
    """A key: non-empty, relative, ``/``-separated, no empty / ``.`` / ``..`` segments, NUL or backslash."""

    _require(isinstance(key, str) and bool(key), f"{label} must be a non-empty string")
    assert isinstance(key, str)
    _require("\x00" not in key and "\\" not in key, f"{label} must not contain NUL or backslash: {key!r}")
    segments = key.split("/")
    _require(all(s not in ("", ".", "..") for s in segments),
             f"{label} must be relative, without empty, '.' or '..' segments: {key!r}")
    _require(all(_TEMP_MARKER not in s for s in segments), f"{label} must not contain {_TEMP_MARKER!r}: {key!r}")
    return key


def _prefix(prefix: object) -> str:
    """A listing prefix: empty, or a key optionally ending in ``/``."""

    if prefix == "":
        return ""
    _require(isinstance(prefix, str), "prefix must be a string")
    assert isinstance(prefix, str)
    validate_key(prefix.removesuffix("/"), "prefix")
    return prefix


def _byte_range(offset: object, length: object) -> None:
    _require(type(offset) is int and offset >= 0, "offset must be a non-negative integer")
    _require(length is None or (type(length) is int and length >= 0),
             "length must be a non-negative integer or None")


def _pieces(data: PutData) -> Iterator[Union[bytes, bytearray, memoryview]]:
    if isinstance(data, (bytes, bytearray, memoryview)):
        yield data
        return
    _require(not isinstance(data, str), "put data must be bytes or an iterable of bytes, not str", TypeError)
    for piece in data:
        _require(isinstance(piece, (bytes, bytearray, memoryview)),
                 f"put data chunks must be bytes-like, got {type(piece).__name__}", TypeError)
        yield piece


def _size_and_digest(path: str) -> Tuple[int, str]:
    h = hashlib.sha256()
    size = 0
    with open(path, "rb") as fh:
        for block in iter(lambda: fh.read(_BLOCK), b""):
            h.update(block)
            size += len(block)
    return size, h.hexdigest()


def transient_read_error(error: BaseException) -> bool:
    return isinstance(error, OSError) and error.errno in _TRANSIENT


# ----------------------------------------------------------------------------- local store


def _stream_into(fh: BinaryIO, data: PutData, sync: bool) -> Tuple[int, str]:
    h = hashlib.sha256()
    size = 0
    for piece in _pieces(data):
        fh.write(piece)
        h.update(piece)
        size += len(piece)
    fh.flush()
    if sync:
        os.fsync(fh.fileno())
    return size, h.hexdigest()


def _publish_by_link(path: str, data: PutData, sync: bool, mode: int, root: str) -> Tuple[int, str]:
    directory, name = os.path.split(path)
    fd, staging = tempfile.mkstemp(prefix=f".{name}{_TEMP_MARKER}", dir=directory)
    try:
        with os.fdopen(fd, "wb") as fh:
            written = _stream_into(fh, data, sync)
        os.chmod(staging, mode)
        try:
            os.link(staging, path)  # FileExistsError: the key exists and stays as it was
        except FileExistsError:
            raise
        except OSError as exc:
            if exc.errno in _NO_HARDLINK:
                raise OSError(exc.errno, f"{root} does not support hard links; use "
                                         "LocalStore(..., publish='exclusive') on this mount") from exc
            raise
        return written
    finally:
        try:
            os.unlink(staging)
        except FileNotFoundError:
            pass


def _publish_exclusive(path: str, data: PutData, sync: bool, mode: int, root: str) -> Tuple[int, str]:
    flags = os.O_WRONLY | os.O_CREAT | os.O_EXCL | getattr(os, "O_NOFOLLOW", 0) | getattr(os, "O_CLOEXEC", 0)
    fd = os.open(path, flags, mode)
    try:
        with os.fdopen(fd, "wb") as fh:
            return _stream_into(fh, data, sync)
    except BaseException:
        try:
            os.unlink(path)  # created by this call: the partial object is ours to remove
        except FileNotFoundError:
            pass
        raise


_PUBLISHERS = {"link": _publish_by_link, "exclusive": _publish_exclusive}


def _non_negative_seconds(value: Any, name: str) -> float:
    seconds = float(value)
    _require(math.isfinite(seconds) and seconds >= 0, f"{name} must be a finite, non-negative number")
    return seconds


class LocalStore:
    """A store over a POSIX directory tree (see the module notes for the two publication modes)."""

    def __init__(self, root: Union[str, "os.PathLike[str]"], *, publish: str = "link", fsync: bool = True,
                 verify_readback: bool = False, settle_seconds: float = 0.0, file_mode: int = 0o444,
                 profile: Optional[StoreProfile] = None, read_settle_seconds: float = 0.0) -> None:
        _require(publish in _PUBLISHERS, f"publish must be one of {tuple(_PUBLISHERS)}, got {publish!r}")
        _require(isinstance(fsync, bool) and isinstance(verify_readback, bool),
                 "fsync and verify_readback must be booleans")
        self.settle_seconds = _non_negative_seconds(settle_seconds, "settle_seconds")
        _require(self.settle_seconds == 0 or verify_readback, "settle_seconds requires verify_readback=True")
        _require(type(file_mode) is int and 0 <= file_mode <= 0o777,
                 "file_mode must be a permission mode between 0 and 0o777")
        self.read_settle_seconds = _non_negative_seconds(read_settle_seconds, "read_settle_seconds")
        _require(profile is None or isinstance(profile, StoreProfile), "profile must be a StoreProfile", TypeError)
        self.root = canonical_dir(os.fspath(root))
        self.publish, self.fsync, self.verify_readback, self.file_mode = publish, fsync, verify_readback, file_mode
        self.profile = profile or LOCAL_PROFILE

    def __repr__(self) -> str:
        return (f"LocalStore({self.root!r}, publish={self.publish!r}, fsync={self.fsync}, "
                f"verify_readback={self.verify_readback}, settle_seconds={self.settle_seconds})")

    def _path(self, key: str) -> str:
        return os.path.join(self.root, *validate_key(key).split("/"))

    def _patiently(self, action: Callable[[], Any]) -> Any:
        """Run a read, retrying transient errors until ``read_settle_seconds`` have passed."""

        give_up = time.monotonic() + self.read_settle_seconds
        while True:
            try:
                return action()
            except OSError as exc:
                left = give_up - time.monotonic()
                if exc.errno not in _TRANSIENT or left <= 0:
                    raise
                time.sleep(min(5.0, left))

    def get(self, key: str, offset: int = 0, length: Optional[int] = None) -> bytes:
        _byte_range(offset, length)
        path = self._path(key)

        def read() -> bytes:
            with open(path, "rb") as fh:
                fh.seek(offset)
                return fh.read(-1 if length is None else length)

        return self._patiently(read)

    def open(self, key: str) -> BinaryIO:
        path = self._path(key)
        return self._patiently(lambda: open(path, "rb"))

    def put(self, key: str, data: PutData) -> ObjectInfo:
        path = self._path(key)
        directory = os.path.dirname(path)
        os.makedirs(directory, exist_ok=True)
        size, digest = _PUBLISHERS[self.publish](path, data, self.fsync, self.file_mode, self.root)
        if self.fsync:
            _fsync_directory(directory)
        if self.verify_readback:
            self._confirm(path, size, digest)
        return ObjectInfo(key, size, digest)

    def _confirm(self, path: str, size: int, digest: str) -> None:
        """Re-read until the object has the written size and digest, for up to ``settle_seconds``."""

        give_up = time.monotonic() + self.settle_seconds
        problem: Optional[OSError] = None
        while True:
            try:
                if _size_and_digest(path) == (size, digest):
                    return
            except OSError as exc:
                problem = exc
            left = give_up - time.monotonic()
            if left <= 0:
                detail = "" if problem is None else f" (last error: {problem})"
                raise OSError(f"{path} did not read back with the written size and SHA256 within "
                              f"{self.settle_seconds}s{detail}")
            time.sleep(min(1.0, left))

    def stat(self, key: str) -> Optional[ObjectInfo]:
        path = self._path(key)
        try:
            st = self._patiently(lambda: os.stat(path))
        except (FileNotFoundError, NotADirectoryError):
            return None
        return ObjectInfo(key, st.st_size) if stat.S_ISREG(st.st_mode) else None

    def list(self, prefix: str = "") -> List[str]:
        prefix = _prefix(prefix)
        folder = prefix.rpartition("/")[0]
        start = os.path.join(self.root, *folder.split("/")) if folder else self.root
        if not os.path.isdir(start):
            return []
        found: List[str] = []
        for directory, subdirs, files in os.walk(start):
            rel = os.path.relpath(directory, self.root)
            here = "" if rel == "." else rel.replace(os.sep, "/") + "/"
            # Descend only where keys with this prefix can live.
            subdirs[:] = [d for d in subdirs if (here + d).startswith(prefix) or prefix.startswith(here + d + "/")]
            found += [here + f for f in files
                      if (here + f).startswith(prefix) and not (f.startswith(".") and _TEMP_MARKER in f)]
        return sorted(found)

    def delete(self, key: str) -> None:
        try:
            os.remove(self._path(key))
        except FileNotFoundError:
            pass

    def local_path(self, key: str) -> Optional[str]:
        return self._path(key)


# ----------------------------------------------------------------------------- registry


_SCHEME = re.compile(r"[a-z][a-z0-9+.-]*")


def validate_scheme(scheme: object) -> str:
    _require(isinstance(scheme, str) and _SCHEME.fullmatch(scheme) is not None, f"invalid store scheme {scheme!r}")
    _require(scheme != "file", "the 'file' scheme is built in")
    assert isinstance(scheme, str)
    return scheme


class StoreRegistry:
    """Factories for ``scheme://`` stores: registered in-process or found through entry points."""

    def __init__(self) -> None:
        self.factories: Dict[str, StoreFactory] = {}

    def register(self, scheme: str, factory: StoreFactory) -> None:
        validate_scheme(scheme)
        _require(callable(factory), "store factory must be callable", TypeError)
        existing = self.factories.setdefault(scheme, factory)
        _require(existing is factory, f"store scheme {scheme!r} is already registered")

    @staticmethod
    def _entry_points() -> list:
        return list(metadata.entry_points(group=ENTRY_POINT_GROUP))

    def provides(self, scheme: str) -> bool:
        return scheme in self.factories or any(ep.name == scheme for ep in self._entry_points())

    def factory(self, scheme: str, also_known: Iterable[str] = ()) -> StoreFactory:
        if scheme in self.factories:
            return self.factories[scheme]
        points = self._entry_points()
        providers = [ep for ep in points if ep.name == scheme]
        if not providers:
            known = sorted({"file", *self.factories, *(ep.name for ep in points), *also_known})
            raise ValueError(f"no store is registered for scheme {scheme!r}; known schemes: {known}")
        _require(len(providers) == 1, f"several installed packages provide store scheme {scheme!r}: "
                                      f"{sorted(ep.value for ep in providers)}")
        found = providers[0].load()
        self.register(scheme, found)
        return found


_REGISTRY = StoreRegistry()


def register_store(scheme: str, factory: StoreFactory) -> None:
    _REGISTRY.register(scheme, factory)


def _uri_key_path(location: str) -> str:
    """The part of ``scheme://path`` after the scheme, as a key (``""`` for the store's root)."""

    rest = location.split("://", 1)[1]
    _require("?" not in rest and "#" not in rest, f"store URIs take no query or fragment: {location!r}")
    rest = rest.removesuffix("/")
    return validate_key(unquote(rest), "store URI path") if rest else ""


def _local_from_file_uri(text: str) -> LocalStore:
    parts = urlparse(text)
    _require(parts.netloc in ("", "localhost") and not (parts.params or parts.query or parts.fragment),
             f"file URIs must be file:///absolute/path, got {text!r}")
    return LocalStore(unquote(parts.path))


def open_store(location: Union[str, "os.PathLike[str]", Store], *,
               stores_file: Optional[Union[str, "os.PathLike[str]"]] = None) -> Store:
    """The store at ``location`` (a store object is returned as it is)."""

    if isinstance(location, Store):
        return location
    text = os.fspath(location)
    _require(isinstance(text, str) and bool(text), "store location must be a non-empty string or path")
    if "://" not in text:
        return LocalStore(text)
    scheme = urlparse(text).scheme.lower()
    if scheme == "file":
        return _local_from_file_uri(text)
    from .stores_file import load_default_or_given

    defined = load_default_or_given(stores_file)
    if scheme in defined:
        _require(not _REGISTRY.provides(scheme),
                 f"store scheme {scheme!r} is defined by both the stores file and a plugin")
        return defined[scheme].open(_uri_key_path(text))
    made = _REGISTRY.factory(scheme, defined)(text)
    _require(isinstance(made, Store), f"store factory for {scheme!r} returned {type(made).__name__}, "
                                      "which is not a Store", TypeError)
    return made
