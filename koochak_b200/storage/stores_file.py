"""Named stores from a private YAML file.

(behaviour of reference koochak/storage/stores_file.py:52-185)

Format (a contract shared with the reference)::

    version: 1
    stores:
      scratch: {type: local, root: /abs/path/${oc.env:USER}, publish: link,
                profile: {request_seconds: 0.001, stream_mb_s: 1000, part_bytes: 16MiB}}

The file is ``$KOOCHAK_STORES`` when set, else
``$XDG_CONFIG_HOME/koochak/stores.yaml`` (``~/.config`` by default) when it
exists. ``${oc.env:VAR}`` references are resolved, every entry is checked
against ``_ENTRY_SCHEMA`` (unknown keys fail) and opened once at load time,
and a parsed file is reused until its mtime or size changes.
"""

from __future__ import annotations

import dataclasses
import math
import os
from dataclasses import dataclass
from typing import Any, Callable, Dict, Mapping, Optional, Tuple, Union

from ..utils.sizes import parse_size
from .store import LocalStore, StoreProfile, validate_scheme

__all__ = ["ENV_VAR", "StoreSpec", "default_stores_path", "load_default_or_given", "load_stores_file"]

ENV_VAR = "KOOCHAK_STORES"
VERSION = 1
_PROFILE_FIELDS = frozenset(f.name for f in dataclasses.fields(StoreProfile))
_PARSED: Dict[str, Tuple[int, int, Dict[str, "StoreSpec"]]] = {}


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
        where = os.path.join(self.root, *subpath.split("/")) if subpath else self.root
        return LocalStore(where, publish=self.publish, fsync=self.fsync, verify_readback=self.verify_readback,
                          settle_seconds=self.settle_seconds, profile=self.profile,
                          read_settle_seconds=self.read_settle_seconds)


def default_stores_path() -> Optional[str]:
    if os.environ.get(ENV_VAR):
        return os.environ[ENV_VAR]
    config_home = os.environ.get("XDG_CONFIG_HOME") or os.path.join(os.path.expanduser("~"), ".config")
    candidate = os.path.join(config_home, "koochak", "stores.yaml")
    return candidate if os.path.isfile(candidate) else None


def _mapping(value: Any, label: str, allowed: frozenset) -> Mapping:
    if not isinstance(value, Mapping):
        raise ValueError(f"{label} must be a mapping")
    unknown = set(value) - allowed
    if unknown:
        raise ValueError(f"{label} has unknown keys {sorted(unknown)}; allowed: {sorted(allowed)}")
    return value


def _boolean(value: Any, label: str) -> bool:
    if not isinstance(value, bool):
        raise ValueError(f"{label} must be true or false")
    return value


def _seconds(value: Any, label: str) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
        raise ValueError(f"{label} must be a number")
    return float(value)


def _root(value: Any, label: str) -> str:
    if not isinstance(value, str) or not value or not os.path.isabs(os.path.expanduser(value)):
        raise ValueError(f"{label} must be an absolute path")
    return os.path.abspath(os.path.expanduser(value))


def _kind(value: Any, label: str) -> str:
    if value != "local":
        raise ValueError(f"{label} must be 'local' (the only backend type so far)")
    return value


def _profile(value: Any, label: str) -> StoreProfile:
    fields = dict(_mapping(value, label, _PROFILE_FIELDS))
    if "part_bytes" in fields:
        fields["part_bytes"] = parse_size(fields["part_bytes"])
    return StoreProfile(**fields)


# entry key -> (StoreSpec field, default, parser); a None default means the key is required
_ENTRY_SCHEMA: Dict[str, Tuple[Optional[str], Any, Callable[[Any, str], Any]]] = {
    "type": (None, None, _kind),
    "root": ("root", None, _root),
    "publish": ("publish", "link", lambda v, label: str(v)),
    "fsync": ("fsync", True, _boolean),
    "verify_readback": ("verify_readback", False, _boolean),
    "settle_seconds": ("settle_seconds", 0.0, _seconds),
    "read_settle_seconds": ("read_settle_seconds", 0.0, _seconds),
    "profile": ("profile", dataclasses.MISSING, _profile),
}


def _spec(scheme: str, entry: Any, source: str) -> StoreSpec:
    label = f"{source}: stores.{scheme}"
    entry = _mapping(entry, label, frozenset(_ENTRY_SCHEMA))
    fields: Dict[str, Any] = {"scheme": scheme}
    for key, (field, default, parse) in _ENTRY_SCHEMA.items():
        if key not in entry and default is dataclasses.MISSING:
            continue
        value = entry.get(key, default)
        parsed = parse(value, f"{label}.{key}")
        if field is not None:
            fields[field] = parsed
    return StoreSpec(**fields)


def _read_yaml(path: str) -> Any:
    import yaml

    from ..config import resolve, to_container

    with open(path, encoding="utf-8") as fh:
        raw = yaml.safe_load(fh)
    return to_container(resolve(raw)) if isinstance(raw, Mapping) else raw


def _parse(path: str) -> Dict[str, StoreSpec]:
    data = _read_yaml(path)
    if not isinstance(data, dict) or set(data) != {"version", "stores"}:
        raise ValueError(f"{path}: a stores file has exactly the keys 'version' and 'stores'")
    if data["version"] != VERSION:
        raise ValueError(f"{path}: unsupported stores file version {data['version']!r}")
    entries = data["stores"]
    if not isinstance(entries, dict) or not entries:
        raise ValueError(f"{path}: 'stores' must be a non-empty mapping")
    specs: Dict[str, StoreSpec] = {}
    for scheme, entry in entries.items():
        try:
            validate_scheme(scheme)
        except ValueError as exc:
            raise ValueError(f"{path}: {exc}") from exc
        spec = _spec(scheme, entry, path)
        spec.open()  # a bad combination of options fails here, not at first use
        specs[scheme] = spec
    return specs


def load_stores_file(path: Union[str, "os.PathLike[str]"]) -> Dict[str, StoreSpec]:
    where = os.path.abspath(os.path.expanduser(os.fspath(path)))
    if not os.path.isfile(where):
        raise FileNotFoundError(f"stores file not found: {where}")
    st = os.stat(where)
    cached = _PARSED.get(where)
    if cached is None or cached[:2] != (st.st_mtime_ns, st.st_size):
        cached = (st.st_mtime_ns, st.st_size, _parse(where))
        _PARSED[where] = cached
    return dict(cached[2])


def load_default_or_given(stores_file: Optional[Union[str, "os.PathLike[str]"]] = None) -> Dict[str, StoreSpec]:
    where = default_stores_path() if stores_file is None else stores_file
    return load_stores_file(where) if where is not None else {}
