"""Named stores from a private YAML file (reference: koochak/storage/stores_file.py:52-185).

File format::

    version: 1
    stores:
      scratch: {type: local, root: /abs/path/${oc.env:USER}, publish: link,
                profile: {request_seconds: 0.001, stream_mb_s: 1000, part_bytes: 16MiB}}

The file is ``$KOOCHAK_STORES`` when set, else ``$XDG_CONFIG_HOME/koochak/stores.yaml``
(default ``~/.config``) when it exists. ``${oc.env:VAR}`` is resolved; unknown
keys fail; parsed files are cached until their mtime or size changes.
"""

from __future__ import annotations

import dataclasses
import math
import os
from dataclasses import dataclass
from typing import Any, Dict, Mapping, Optional, Union

from ..utils.sizes import parse_size
from .store import LocalStore, StoreProfile, validate_scheme

__all__ = ["ENV_VAR", "StoreSpec", "default_stores_path", "load_default_or_given", "load_stores_file"]

ENV_VAR = "KOOCHAK_STORES"
VERSION = 1
_ENTRY_KEYS = frozenset({"type", "root", "publish", "fsync", "verify_readback", "settle_seconds",
                         "read_settle_seconds", "profile"})
_PROFILE_KEYS = frozenset(f.name for f in dataclasses.fields(StoreProfile))
_CACHE: Dict[str, tuple] = {}


@dataclass(frozen=True, slots=True)
class StoreSpec:
    scheme: str
    root: str
    publish: str = "link"
    fsync: bool = True
    verify_readback: bool = False
    settle_seconds: float = 0.0
    profile: Optional[StoreProfile] = None
    read_settle_seconds: float = 0.0

    def open(self, subpath: str = "") -> LocalStore:
        root = os.path.join(self.root, *subpath.split("/")) if subpath else self.root
        return LocalStore(root, publish=self.publish, fsync=self.fsync, verify_readback=self.verify_readback,
                          settle_seconds=self.settle_seconds, profile=self.profile,
                          read_settle_seconds=self.read_settle_seconds)


def default_stores_path() -> Optional[str]:
    explicit = os.environ.get(ENV_VAR)
    if explicit:
        return explicit
    base = os.environ.get("XDG_CONFIG_HOME") or os.path.join(os.path.expanduser("~"), ".config")
    path = os.path.join(base, "koochak", "stores.yaml")
    return path if os.path.isfile(path) else None


def _bool(v: object, label: str) -> bool:
    if not isinstance(v, bool):
        raise ValueError(f"{label} must be true or false")
    return v


def _profile(v: object, label: str) -> StoreProfile:
    if not isinstance(v, Mapping):
        raise ValueError(f"{label} must be a mapping")
    extra = set(v) - _PROFILE_KEYS
    if extra:
        raise ValueError(f"{label} has unknown keys {sorted(extra)}; allowed: {sorted(_PROFILE_KEYS)}")
    kw = dict(v)
    if "part_bytes" in kw:
        kw["part_bytes"] = parse_size(kw["part_bytes"])
    return StoreProfile(**kw)


def _spec(scheme: str, v: object, source: str) -> StoreSpec:
    label = f"{source}: stores.{scheme}"
    if not isinstance(v, Mapping):
        raise ValueError(f"{label} must be a mapping")
    extra = set(v) - _ENTRY_KEYS
    if extra:
        raise ValueError(f"{label} has unknown keys {sorted(extra)}; allowed: {sorted(_ENTRY_KEYS)}")
    if v.get("type") != "local":
        raise ValueError(f"{label}.type must be 'local' (the only backend type so far)")
    root = v.get("root")
    if not isinstance(root, str) or not root or not os.path.isabs(os.path.expanduser(root)):
        raise ValueError(f"{label}.root must be an absolute path")
    settle, read_settle = v.get("settle_seconds", 0.0), v.get("read_settle_seconds", 0.0)
    for name, num in (("settle_seconds", settle), ("read_settle_seconds", read_settle)):
        if isinstance(num, bool) or not isinstance(num, (int, float)) or not math.isfinite(num):
            raise ValueError(f"{label}.{name} must be a number")
    return StoreSpec(scheme=scheme, root=os.path.abspath(os.path.expanduser(root)),
                     publish=str(v.get("publish", "link")), fsync=_bool(v.get("fsync", True), f"{label}.fsync"),
                     verify_readback=_bool(v.get("verify_readback", False), f"{label}.verify_readback"),
                     settle_seconds=float(settle),
                     profile=_profile(v["profile"], f"{label}.profile") if "profile" in v else None,
                     read_settle_seconds=float(read_settle))


def _load_yaml_resolved(path: str) -> Any:
    import yaml

    from ..config import resolve, to_container

    with open(path, encoding="utf-8") as fh:
        data = yaml.safe_load(fh)
    return to_container(resolve(data)) if isinstance(data, Mapping) else data


def load_stores_file(path: Union[str, "os.PathLike[str]"]) -> Dict[str, StoreSpec]:
    absolute = os.path.abspath(os.path.expanduser(os.fspath(path)))
    if not os.path.isfile(absolute):
        raise FileNotFoundError(f"stores file not found: {absolute}")
    st = os.stat(absolute)
    hit = _CACHE.get(absolute)
    if hit is not None and hit[:2] == (st.st_mtime_ns, st.st_size):
        return dict(hit[2])
    data = _load_yaml_resolved(absolute)
    if not isinstance(data, dict) or set(data) != {"version", "stores"}:
        raise ValueError(f"{absolute}: a stores file has exactly the keys 'version' and 'stores'")
    if data["version"] != VERSION:
        raise ValueError(f"{absolute}: unsupported stores file version {data['version']!r}")
    stores = data["stores"]
    if not isinstance(stores, dict) or not stores:
        raise ValueError(f"{absolute}: 'stores' must be a non-empty mapping")
    specs: Dict[str, StoreSpec] = {}
    for scheme, v in stores.items():
        try:
            validate_scheme(scheme)
        except ValueError as exc:
            raise ValueError(f"{absolute}: {exc}") from exc
        specs[scheme] = _spec(scheme, v, absolute)
        specs[scheme].open()  # invalid combinations fail now, not at first use
    _CACHE[absolute] = (st.st_mtime_ns, st.st_size, specs)
    return dict(specs)


def load_default_or_given(stores_file: Optional[Union[str, "os.PathLike[str]"]] = None) -> Dict[str, StoreSpec]:
    path = stores_file if stores_file is not None else default_stores_path()
    return {} if path is None else load_stores_file(path)
