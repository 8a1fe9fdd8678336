"""Checkpoint publication and auto-resume (reference: koochak/storage/checkpoint.py:74-459).

On-disk format (kept byte-compatible with the reference):

* ``step{N:09d}.pt``: ``torch.save`` bytes of the checkpoint dict, written
  create-only through a :class:`Store`;
* ``step{N:09d}.pt.ready.json``: written after the payload and therefore its
  commit point: canonical JSON (sorted keys, ``,``/``:`` separators, trailing
  newline) of exactly ``{v, artifact_id, path, size_bytes, sha256, manifest_path}``;
* ``latest.pt``: a symlink, only for hard-link (``publish="link"``) stores.

Resume trusts a numbered checkpoint only when its manifest, size and SHA-256
agree with the payload bytes it then loads.
"""

from __future__ import annotations

import hashlib
import io
import json
import os
import pickle
import re
import shutil
from collections import OrderedDict
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple, Union

import torch

from ..utils.paths import canonical_dir
from . import fs as fs_utils
from .store import LocalStore, Store, open_store

__all__ = ["BackgroundPublisher", "add_module_prefix", "best", "checkpoint_path", "checkpoint_store",
           "highest_valid_published", "latest_valid", "latest", "load", "match_state_dict_to_model", "prune",
           "publication", "publication_path", "publish", "resolve_auto_resume", "save", "serialize",
           "strip_module_prefix", "PUBLICATION_SUFFIX", "AutoResumeSelection"]

PUBLICATION_SUFFIX = ".ready.json"
_NUMBERED = re.compile(r"step(\d+)\.pt")
_STEP_RE = re.compile(r"step(\d+)\.pt$")
_MANIFEST_KEYS = frozenset({"v", "artifact_id", "path", "size_bytes", "sha256", "manifest_path"})
_ABSENT = (FileNotFoundError, IsADirectoryError, NotADirectoryError)
_CORRUPT = (EOFError, RuntimeError, ValueError, TypeError, AttributeError, IndexError, KeyError, ImportError,
            MemoryError, OverflowError, pickle.PickleError)

Location = Union[str, "os.PathLike[str]", Store]


@dataclass(frozen=True, slots=True)
class AutoResumeSelection:
    path: str
    checkpoint: Dict[str, Any]
    next_step: int


def serialize(ckpt: Dict[str, Any]) -> bytes:
    buf = io.BytesIO()
    torch.save(ckpt, buf)
    return buf.getvalue()


def checkpoint_store(location: Location) -> Store:
    """Directory -> owner-only LocalStore; ``scheme://`` -> configured store; a Store as-is."""

    if isinstance(location, Store):
        return location
    text = os.fspath(location)
    if "://" in text:
        return open_store(text)
    return LocalStore(canonical_dir(text), file_mode=0o600)


def checkpoint_path(store: Store, name: str) -> str:
    path = store.local_path(name)
    if path is None:
        raise TypeError(f"{store!r} exposes no filesystem paths; checkpoint stores must be filesystem-backed")
    return path


def publication_path(path: str) -> str:
    return os.path.abspath(path) + PUBLICATION_SUFFIX


def _manifest(path: str, size: int, sha256: str) -> dict[str, Any]:
    absolute = os.path.abspath(path)
    return {"v": 1, "artifact_id": f"checkpoint/{os.path.basename(absolute)}", "path": absolute,
            "size_bytes": size, "sha256": sha256, "manifest_path": publication_path(absolute)}


def _encode_manifest(record: dict[str, Any]) -> bytes:
    return (json.dumps(record, sort_keys=True, separators=(",", ":"), ensure_ascii=False) + "\n").encode("utf-8")


def publication(path: str) -> dict[str, Any]:
    mpath = publication_path(path)
    with open(mpath, encoding="utf-8") as fh:
        record = json.load(fh)
    if not isinstance(record, dict) or set(record) != _MANIFEST_KEYS or record.get("v") != 1:
        raise ValueError(f"invalid checkpoint publication manifest: {mpath}")
    return record


def _copy_as_latest(step_path: str, latest_path: str) -> Optional[str]:
    try:
        shutil.copy2(step_path, latest_path)
        return latest_path
    except OSError:
        return None


def _refresh_latest_link(step_path: str) -> Optional[str]:
    directory = os.path.dirname(os.path.abspath(step_path))
    latest_path = os.path.join(directory, "latest.pt")
    if os.path.islink(latest_path) or os.path.exists(latest_path):
        try:
            os.remove(latest_path)
        except FileNotFoundError:
            pass
        except OSError:
            return _copy_as_latest(step_path, latest_path)
    try:
        os.symlink(os.path.basename(step_path), latest_path)
        return latest_path
    except (OSError, NotImplementedError):
        return _copy_as_latest(step_path, latest_path)


def _numbered(store: Store) -> List[Tuple[int, str]]:
    out = []
    for key in store.list("step"):
        m = _NUMBERED.fullmatch(key)
        if m:
            out.append((int(m.group(1)), key))
    return sorted(out)


def _validated(store: Store, name: str) -> Optional[AutoResumeSelection]:
    """The checkpoint behind ``name`` if its manifest, size, digest and cursor all agree."""

    m = _NUMBERED.fullmatch(name)
    if m is None:
        return None
    absolute = os.path.abspath(checkpoint_path(store, name))
    mpath = publication_path(absolute)
    try:
        if any(not os.path.isfile(p) or os.path.islink(p) for p in (absolute, mpath)):
            return None
        record = json.loads(store.get(name + PUBLICATION_SUFFIX).decode("utf-8"))
        if not isinstance(record, dict) or set(record) != _MANIFEST_KEYS or record["v"] != 1:
            return None
        if record["artifact_id"] != f"checkpoint/{name}" or record["path"] != absolute \
                or record["manifest_path"] != mpath:
            return None
        info = store.stat(name)
        if info is None or type(record["size_bytes"]) is not int or record["size_bytes"] != info.size:
            return None
        payload = store.get(name)
        if len(payload) != info.size or record["sha256"] != hashlib.sha256(payload).hexdigest():
            return None
        ckpt = torch.load(io.BytesIO(payload), weights_only=False, map_location="cpu")
        if not isinstance(ckpt, dict):
            return None
        step, nxt = ckpt.get("step"), ckpt.get("next_step")
        if type(step) is not int or type(nxt) is not int or nxt < 0 or step != int(m.group(1)):
            return None
        if nxt not in (step, step + 1):  # periodic (step+1) or terminal (step)
            return None
    except _ABSENT:
        return None
    except _CORRUPT:
        return None
    return AutoResumeSelection(absolute, ckpt, nxt)


def _highest_valid(store: Store) -> Optional[AutoResumeSelection]:
    for _step, key in reversed(_numbered(store)):
        sel = _validated(store, key)
        if sel is not None:
            return sel
    return None


def highest_valid_published(location: Location) -> Optional[str]:
    sel = _highest_valid(checkpoint_store(location))
    return None if sel is None else sel.path


latest_valid = highest_valid_published


def resolve_auto_resume(location: Location) -> Optional[tuple[str, Dict[str, Any]]]:
    """``(path, checkpoint)`` of the newest valid published checkpoint, or None."""

    sel = _highest_valid(checkpoint_store(location))
    return None if sel is None else (sel.path, sel.checkpoint)


def prune(store: Store, keep_last_k: int) -> None:
    """Drop all but the newest ``keep_last_k`` numbered checkpoints, manifest first."""

    if keep_last_k <= 0:
        return
    for _step, key in _numbered(store)[:-keep_last_k]:
        store.delete(key + PUBLICATION_SUFFIX)
        store.delete(key)


def publish(store: Store, name: str, data: bytes, *, keep_last_k: int = 3) -> str:
    """Payload create-only, then manifest; replaces a same-named checkpoint (uncommitting it first)."""

    path = checkpoint_path(store, name)
    mname = name + PUBLICATION_SUFFIX
    if store.stat(name) is not None or store.stat(mname) is not None:
        store.delete(mname)
        store.delete(name)
    info = store.put(name, data)
    digest = info.sha256 if info.sha256 is not None else hashlib.sha256(data).hexdigest()
    store.put(mname, _encode_manifest(_manifest(path, info.size, digest)))
    if isinstance(store, LocalStore) and store.publish == "link":
        _refresh_latest_link(path)
    prune(store, keep_last_k)
    return path


def save(ckpt: Dict[str, Any], path: str, keep_last_k: int = 3) -> str:
    directory = os.path.dirname(os.path.abspath(path)) or "."
    publish(checkpoint_store(directory), os.path.basename(path), serialize(ckpt), keep_last_k=keep_last_k)
    return path


class BackgroundPublisher:
    """One publication at a time on a background thread.

    ``submit`` returns the path at once; ``poll``/``wait`` return ``(path, token)``
    once committed and re-raise a failed publication on the caller's thread.
    """

    def __init__(self, store: Store, *, keep_last_k: int) -> None:
        self.store = store
        self.keep_last_k = keep_last_k
        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="koochak-checkpoint")
        self._pending: Optional[Tuple[Future, Any]] = None

    @property
    def pending(self) -> bool:
        return self._pending is not None

    def submit(self, name: str, data: bytes, token: Any = None) -> str:
        if self._pending is not None:
            raise RuntimeError("a checkpoint publication is already pending; wait() for it first")
        path = checkpoint_path(self.store, name)
        self._pending = (self._pool.submit(publish, self.store, name, data, keep_last_k=self.keep_last_k), token)
        return path

    def poll(self) -> Optional[Tuple[str, Any]]:
        if self._pending is None or not self._pending[0].done():
            return None
        return self.wait()

    def wait(self) -> Optional[Tuple[str, Any]]:
        if self._pending is None:
            return None
        fut, token = self._pending
        self._pending = None
        return fut.result(), token

    def close(self) -> None:
        self._pool.shutdown(wait=True)
        self._pending = None


def load(path: str) -> Dict[str, Any]:
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    return torch.load(path, weights_only=False, map_location="cpu")


def _directory(location: Location) -> str:
    if isinstance(location, LocalStore):
        return location.root
    text = os.fspath(location)
    if "://" not in text:
        return text
    store = checkpoint_store(text)
    if not isinstance(store, LocalStore):
        raise TypeError(f"{text} does not resolve to a filesystem directory")
    return store.root


def latest(location: Location) -> Optional[str]:
    return fs_utils.latest(_directory(location), pattern=_STEP_RE.pattern)


def best(location: Location, key: str = "val_loss") -> Optional[str]:
    return fs_utils.best(_directory(location), key=key, pattern=_STEP_RE.pattern)


def _all_prefixed(sd: Dict[str, Any]) -> bool:
    keys = list(sd.keys())
    return bool(keys) and all(isinstance(k, str) and k.startswith("module.") for k in keys)


def strip_module_prefix(sd: Dict[str, Any]) -> "OrderedDict[str, Any]":
    return OrderedDict((k[7:] if isinstance(k, str) and k.startswith("module.") else k, v) for k, v in sd.items())


def add_module_prefix(sd: Dict[str, Any]) -> "OrderedDict[str, Any]":
    return OrderedDict((f"module.{k}" if isinstance(k, str) and not k.startswith("module.") else k, v)
                       for k, v in sd.items())


def match_state_dict_to_model(model: Any, sd: Dict[str, Any]) -> "OrderedDict[str, Any]":
    """Add or strip the DDP ``module.`` prefix so ``sd`` matches ``model``'s keys."""

    fn = getattr(model, "state_dict", None)
    if fn is None:
        return OrderedDict(sd)
    wants = any(isinstance(k, str) and k.startswith("module.") for k in fn().keys())
    has = _all_prefixed(sd)
    if wants and not has:
        return add_module_prefix(sd)
    if has and not wants:
        return strip_module_prefix(sd)
    return OrderedDict(sd)
