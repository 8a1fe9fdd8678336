"""Checkpoint publication, validation and auto-resume.

(behaviour of reference koochak/storage/checkpoint.py:74-459)

On-disk format, shared with the reference so either framework resumes the
other's runs:

* ``step{N:09d}.pt`` -- ``torch.save`` bytes of the checkpoint dict, put
  create-only through a ``Store``;
* ``step{N:09d}.pt.ready.json`` -- the commit point, written after the
  payload: canonical JSON (sorted keys, ``,``/``:`` separators, trailing
  newline) of exactly ``{v, artifact_id, path, size_bytes, sha256,
  manifest_path}`` (``_Manifest``);
* ``latest.pt`` -- a symlink to the newest payload, only on hard-link
  (``publish="link"``) local stores.

A numbered checkpoint is trusted for resume only when its manifest names it,
its size and SHA-256 match the bytes, those bytes load as a dict, and its
``step`` / ``next_step`` cursor agrees with the file name
(``_verify``). Pruning removes the manifest before the payload, so a
half-pruned checkpoint is never mistaken for a valid one.
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
_STEP_NAME = re.compile(r"step(\d+)\.pt")
_STEP_PATTERN = r"step(\d+)\.pt$"
# Errors that mean "this candidate is not usable", not "resume failed".
_UNUSABLE = (FileNotFoundError, IsADirectoryError, NotADirectoryError, EOFError, RuntimeError, ValueError, TypeError,
             AttributeError, IndexError, KeyError, ImportError, MemoryError, OverflowError, pickle.PickleError)

Location = Union[str, "os.PathLike[str]", Store]


@dataclass(frozen=True, slots=True)
class AutoResumeSelection:
    path: str
    checkpoint: Dict[str, Any]
    next_step: int


@dataclass(frozen=True)
class _Manifest:
    """The ``.ready.json`` record of one published checkpoint payload."""

    path: str
    size_bytes: int
    sha256: str

    FIELDS = frozenset({"v", "artifact_id", "path", "size_bytes", "sha256", "manifest_path"})

    @classmethod
    def for_payload(cls, path: str, size: int, sha256: str) -> "_Manifest":
        return cls(os.path.abspath(path), int(size), sha256)

    def record(self) -> Dict[str, Any]:
        return {"v": 1, "artifact_id": f"checkpoint/{os.path.basename(self.path)}", "path": self.path,
                "size_bytes": self.size_bytes, "sha256": self.sha256, "manifest_path": publication_path(self.path)}

    def encode(self) -> bytes:
        text = json.dumps(self.record(), sort_keys=True, separators=(",", ":"), ensure_ascii=False)
        return (text + "\n").encode("utf-8")

    @classmethod
    def well_formed(cls, record: Any) -> bool:
        return isinstance(record, dict) and set(record) == cls.FIELDS and record.get("v") == 1


def serialize(ckpt: Dict[str, Any]) -> bytes:
    out = io.BytesIO()
    torch.save(ckpt, out)
    return out.getvalue()


def checkpoint_store(location: Location) -> Store:
    """A store for checkpoints: a directory becomes an owner-only ``LocalStore``, a URI its configured store."""

    if isinstance(location, Store):
        return location
    text = os.fspath(location)
    return open_store(text) if "://" in text else LocalStore(canonical_dir(text), file_mode=0o600)


def checkpoint_path(store: Store, name: str) -> str:
    found = store.local_path(name)
    if found is None:
        raise TypeError(f"{store!r} exposes no filesystem paths; checkpoint stores must be filesystem-backed")
    return found


def publication_path(path: str) -> str:
    return os.path.abspath(path) + PUBLICATION_SUFFIX


def publication(path: str) -> dict:
    """The manifest of the checkpoint at ``path`` (ValueError when malformed)."""

    where = publication_path(path)
    with open(where, encoding="utf-8") as fh:
        record = json.load(fh)
    if not _Manifest.well_formed(record):
        raise ValueError(f"invalid checkpoint publication manifest: {where}")
    return record


def _point_latest_at(step_path: str) -> Optional[str]:
    """``latest.pt`` -> the new payload (a symlink; a copy where links cannot be made)."""

    link = os.path.join(os.path.dirname(os.path.abspath(step_path)), "latest.pt")

    def copy() -> Optional[str]:
        try:
            shutil.copy2(step_path, link)
            return link
        except OSError:
            return None

    if os.path.lexists(link):
        try:
            os.remove(link)
        except FileNotFoundError:
            pass
        except OSError:
            return copy()
    try:
        os.symlink(os.path.basename(step_path), link)
        return link
    except (OSError, NotImplementedError):
        return copy()


def _steps(store: Store) -> List[Tuple[int, str]]:
    """(step, key) of every numbered payload in the store, oldest first."""

    found = ((_STEP_NAME.fullmatch(k), k) for k in store.list("step"))
    return sorted((int(m.group(1)), k) for m, k in found if m is not None)


def _verify(store: Store, name: str) -> Optional[AutoResumeSelection]:
    """The checkpoint behind ``name`` when manifest, bytes and cursor all agree; otherwise None."""

    numbered = _STEP_NAME.fullmatch(name)
    if numbered is None:
        return None
    payload_path = os.path.abspath(checkpoint_path(store, name))
    manifest_path = publication_path(payload_path)
    try:
        if not all(os.path.isfile(p) and not os.path.islink(p) for p in (payload_path, manifest_path)):
            return None
        record = json.loads(store.get(name + PUBLICATION_SUFFIX).decode("utf-8"))
        expected = {"artifact_id": f"checkpoint/{name}", "path": payload_path, "manifest_path": manifest_path}
        if not _Manifest.well_formed(record) or any(record[k] != v for k, v in expected.items()):
            return None
        info = store.stat(name)
        if info is None or type(record["size_bytes"]) is not int or record["size_bytes"] != info.size:
            return None
        payload = store.get(name)
        if len(payload) != info.size or hashlib.sha256(payload).hexdigest() != record["sha256"]:
            return None
        ckpt = torch.load(io.BytesIO(payload), weights_only=False, map_location="cpu")
        if not isinstance(ckpt, dict):
            return None
        step, nxt = ckpt.get("step"), ckpt.get("next_step")
        cursor_ok = (type(step) is int and type(nxt) is int and step == int(numbered.group(1))
                     and nxt >= 0 and nxt in (step, step + 1))  # periodic (step + 1) or terminal (step)
        return AutoResumeSelection(payload_path, ckpt, nxt) if cursor_ok else None
    except _UNUSABLE:
        return None


def _newest_valid(store: Store) -> Optional[AutoResumeSelection]:
    for _, key in reversed(_steps(store)):
        chosen = _verify(store, key)
        if chosen is not None:
            return chosen
    return None


def highest_valid_published(location: Location) -> Optional[str]:
    chosen = _newest_valid(checkpoint_store(location))
    return chosen.path if chosen else None


latest_valid = highest_valid_published


def resolve_auto_resume(location: Location) -> Optional[tuple]:
    """``(path, checkpoint)`` of the newest valid published checkpoint, or None."""

    chosen = _newest_valid(checkpoint_store(location))
    return (chosen.path, chosen.checkpoint) if chosen else None


def prune(store: Store, keep_last_k: int) -> None:
    """Keep the newest ``keep_last_k`` numbered checkpoints (manifest removed before its payload)."""

    if keep_last_k > 0:
        for _, key in _steps(store)[:-keep_last_k]:
            store.delete(key + PUBLICATION_SUFFIX)
            store.delete(key)


def publish(store: Store, name: str, data: bytes, *, keep_last_k: int = 3) -> str:
    """Put the payload create-only, then its manifest; a same-named checkpoint is uncommitted and replaced."""

    path = checkpoint_path(store, name)
    manifest_key = name + PUBLICATION_SUFFIX
    if store.stat(name) is not None or store.stat(manifest_key) is not None:
        store.delete(manifest_key)  # uncommit first
        store.delete(name)
    info = store.put(name, data)
    manifest = _Manifest.for_payload(path, info.size, info.sha256 or hashlib.sha256(data).hexdigest())
    store.put(manifest_key, manifest.encode())
    if isinstance(store, LocalStore) and store.publish == "link":
        _point_latest_at(path)
    prune(store, keep_last_k)
    return path


def save(ckpt: Dict[str, Any], path: str, keep_last_k: int = 3) -> str:
    where = os.path.dirname(os.path.abspath(path)) or "."
    publish(checkpoint_store(where), os.path.basename(path), serialize(ckpt), keep_last_k=keep_last_k)
    return path


class BackgroundPublisher:
    """Publishes one checkpoint at a time on a worker thread.

    ``submit`` returns the future path at once; ``poll`` (non-blocking) and
    ``wait`` hand back ``(path, token)`` once the manifest is written, and
    re-raise a failed publication on the caller's thread.
    """

    def __init__(self, store: Store, *, keep_last_k: int) -> None:
        self.store = store
        self.keep_last_k = keep_last_k
        self._worker = ThreadPoolExecutor(max_workers=1, thread_name_prefix="koochak-checkpoint")
        self._inflight: Optional[Tuple[Future, Any]] = None

    @property
    def pending(self) -> bool:
        return self._inflight is not None

    def submit(self, name: str, data: bytes, token: Any = None) -> str:
        if self._inflight is not None:
            raise RuntimeError("a checkpoint publication is already pending; wait() for it first")
        future = self._worker.submit(publish, self.store, name, data, keep_last_k=self.keep_last_k)
        self._inflight = (future, token)
        return checkpoint_path(self.store, name)

    def poll(self) -> Optional[Tuple[str, Any]]:
        return self.wait() if self._inflight is not None and self._inflight[0].done() else None

    def wait(self) -> Optional[Tuple[str, Any]]:
        if self._inflight is None:
            return None
        future, token = self._inflight
        self._inflight = None
        return future.result(), token

    def close(self) -> None:
        self._worker.shutdown(wait=True)
        self._inflight = None


def load(path: str) -> Dict[str, Any]:
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    return torch.load(path, weights_only=False, map_location="cpu")


def _directory_of(location: Location) -> str:
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
    return fs_utils.latest(_directory_of(location), pattern=_STEP_PATTERN)


def best(location: Location, key: str = "val_loss") -> Optional[str]:
    return fs_utils.best(_directory_of(location), key=key, pattern=_STEP_PATTERN)


_PREFIX = "module."


def _prefixed(key: Any) -> bool:
    return isinstance(key, str) and key.startswith(_PREFIX)


def strip_module_prefix(sd: Dict[str, Any]) -> "OrderedDict[str, Any]":
    return OrderedDict((k[len(_PREFIX):] if _prefixed(k) else k, v) for k, v in sd.items())


def add_module_prefix(sd: Dict[str, Any]) -> "OrderedDict[str, Any]":
    return OrderedDict((k if _prefixed(k) or not isinstance(k, str) else _PREFIX + k, v) for k, v in sd.items())


def match_state_dict_to_model(model: Any, sd: Dict[str, Any]) -> "OrderedDict[str, Any]":
    """Add or strip the data-parallel ``module.`` prefix so ``sd``'s keys match ``model``'s."""

    if getattr(model, "state_dict", None) is None:
        return OrderedDict(sd)
    model_wrapped = any(_prefixed(k) for k in model.state_dict().keys())
    sd_wrapped = bool(sd) and all(_prefixed(k) for k in sd.keys())
    if model_wrapped and not sd_wrapped:
        return add_module_prefix(sd)
    if sd_wrapped and not model_wrapped:
        return strip_module_prefix(sd)
    return OrderedDict(sd)
