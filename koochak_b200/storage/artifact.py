"""Ready manifests for file and directory outputs of a run.

(reference: koochak/storage/artifact.py:59-371)

A run declares its outputs (``DeclaredOutput``: id, absolute path, kind
``file`` or ``directory``, stage, provenance, expected record count,
metadata). When an output is complete, ``publish_artifact`` hashes it and
writes ``<path>.ready.json`` once (immutable). The manifest schema (version
1) is the coordinator's contract and is kept field for field:

    v, artifact_id, stage, kind, path, manifest_path, size_bytes, sha256,
    counts{expected, observed}, provenance, metadata, created_at
    [, files: [{path, size_bytes, sha256}...]  for directories]

For a directory, ``sha256`` is the SHA-256 of the canonical JSON of the
sorted per-file entries and ``size_bytes`` their total. Files are read with
``read_stable_regular_file``; symlinked directories are refused.
"""

from __future__ import annotations

import hashlib
import json
import os
import stat
from datetime import datetime, timezone
from pathlib import Path, PurePosixPath
from typing import Any, Dict, List, Mapping, Optional, Tuple

from ..jobs_types import freeze_json, thaw_json, validate_json_value
from .immutable import read_stable_regular_file, write_immutable_file

__all__ = ["ARTIFACT_MANIFEST_VERSION", "DeclaredOutput", "artifact_manifest_path", "build_artifact_manifest",
           "publish_artifact", "validate_artifact", "artifact_publication", "validate_artifact_id"]

ARTIFACT_MANIFEST_VERSION = 1
_KINDS = ("file", "directory")
_DECL_KEYS = ("artifact_id", "path", "kind", "stage", "provenance", "expected_records", "metadata")
_MANIFEST_KEYS = {"v", "artifact_id", "stage", "kind", "path", "manifest_path", "size_bytes", "sha256", "counts",
                  "provenance", "metadata", "created_at"}


def validate_artifact_id(value: object, label: str = "artifact_id") -> str:
    if not isinstance(value, str) or not value.strip():
        raise ValueError(f"{label} must be a non-empty string")
    if value != value.strip():
        raise ValueError(f"{label} must not have leading or trailing whitespace")
    if len(value) > 256 or any(ord(c) < 32 for c in value):
        raise ValueError(f"{label} must be at most 256 printable characters")
    return value


def _abs_path(value: object, label: str) -> str:
    if not isinstance(value, str) or not value or "\x00" in value:
        raise ValueError(f"{label} must be a non-empty path without NUL bytes")
    expanded = os.path.expanduser(value)
    if not os.path.isabs(expanded):
        raise ValueError(f"{label} must be absolute")
    return os.path.abspath(expanded)


def _count(value: object, label: str) -> Optional[int]:
    if value is None:
        return None
    if type(value) is not int or value < 0:
        raise ValueError(f"{label} must be a non-negative integer or null")
    return value


class DeclaredOutput:
    """An immutable output declaration, embedded in a prepared launch."""

    __slots__ = _DECL_KEYS

    def __init__(self, artifact_id: str, path: str, *, kind: str = "file", stage: str = "",
                 provenance: Mapping[str, Any] | None = None, expected_records: int | None = None,
                 metadata: Mapping[str, Any] | None = None) -> None:
        if kind not in _KINDS:
            raise ValueError("kind must be 'file' or 'directory'")
        if not isinstance(stage, str) or "\x00" in stage:
            raise ValueError("stage must be a string without NUL bytes")
        for name, v in (("provenance", provenance), ("metadata", metadata)):
            if v is not None and not isinstance(v, Mapping):
                raise ValueError(f"{name} must be a mapping")
        values = {
            "artifact_id": validate_artifact_id(artifact_id), "path": _abs_path(path, "output path"), "kind": kind,
            "stage": stage, "provenance": freeze_json(provenance or {}, "provenance"),
            "expected_records": _count(expected_records, "expected_records"),
            "metadata": freeze_json(metadata or {}, "metadata"),
        }
        for k, v in values.items():
            object.__setattr__(self, k, v)

    def __setattr__(self, name: str, value: object) -> None:
        raise AttributeError("DeclaredOutput is immutable")

    def __repr__(self) -> str:
        return f"DeclaredOutput(artifact_id={self.artifact_id!r}, path={self.path!r}, kind={self.kind!r})"

    def __eq__(self, other: object) -> bool:
        return isinstance(other, DeclaredOutput) and self.to_dict() == other.to_dict()

    def __hash__(self) -> int:
        return hash(json.dumps(self.to_dict(), sort_keys=True))

    def to_dict(self) -> Dict[str, Any]:
        return {"artifact_id": self.artifact_id, "path": self.path, "kind": self.kind, "stage": self.stage,
                "provenance": thaw_json(self.provenance), "expected_records": self.expected_records,
                "metadata": thaw_json(self.metadata)}

    @classmethod
    def from_dict(cls, value: Mapping[str, Any]) -> "DeclaredOutput":
        if not isinstance(value, Mapping) or set(value) != set(_DECL_KEYS):
            raise ValueError("declared output must contain exactly " + ", ".join(sorted(_DECL_KEYS)))
        return cls(value["artifact_id"], value["path"], kind=value["kind"], stage=value["stage"],
                   provenance=value["provenance"], expected_records=value["expected_records"],
                   metadata=value["metadata"])


def artifact_manifest_path(path: str) -> str:
    return os.path.abspath(path) + ".ready.json"


def _file_entry(path: Path, rel: Optional[str] = None) -> Dict[str, Any]:
    try:
        data = read_stable_regular_file(path)
    except (OSError, ValueError) as exc:
        raise ValueError(f"artifact contains an unavailable or unstable file: {path}") from exc
    return {"path": rel or path.name, "size_bytes": len(data), "sha256": hashlib.sha256(data).hexdigest()}


def _dir_snapshot(d: Path) -> Tuple[int, int, int, int]:
    st = os.lstat(d)
    if not stat.S_ISDIR(st.st_mode):
        raise ValueError(f"artifact directory changed while reading: {d}")
    return st.st_dev, st.st_ino, st.st_mtime_ns, st.st_ctime_ns


def _tree_entries(root: Path) -> List[Dict[str, Any]]:
    try:
        _dir_snapshot(root)
    except (OSError, ValueError) as exc:
        raise ValueError(f"artifact directory is unavailable: {root}") from exc
    seen: Dict[Path, Tuple[int, int, int, int]] = {}
    out: List[Dict[str, Any]] = []
    for dirpath, dirnames, filenames in os.walk(root, followlinks=False):
        d = Path(dirpath)
        seen[d] = _dir_snapshot(d)
        for name in dirnames:
            if not stat.S_ISDIR(os.lstat(d / name).st_mode):
                raise ValueError(f"artifact contains a symlinked directory: {d / name}")
        for name in filenames:
            f = d / name
            out.append(_file_entry(f, PurePosixPath(f.relative_to(root).as_posix()).as_posix()))
    for d, snap in seen.items():  # nothing moved underneath the walk
        if _dir_snapshot(d) != snap:
            raise ValueError(f"artifact directory changed while reading: {d}")
    return sorted(out, key=lambda e: e["path"])


def _digest(kind: str, path: Path):
    if kind == "file":
        e = _file_entry(path)
        return e["size_bytes"], e["sha256"], None
    entries = _tree_entries(path)
    canon = json.dumps(entries, sort_keys=True, separators=(",", ":")).encode()
    return sum(int(e["size_bytes"]) for e in entries), hashlib.sha256(canon).hexdigest(), entries


def build_artifact_manifest(output: DeclaredOutput, *, observed_records: int | None = None,
                            created_at: str | None = None) -> Dict[str, Any]:
    observed = _count(observed_records, "observed_records")
    if output.expected_records is not None and observed != output.expected_records:
        raise ValueError("observed_records must equal expected_records")
    size, digest, entries = _digest(output.kind, Path(output.path))
    m: Dict[str, Any] = {
        "v": ARTIFACT_MANIFEST_VERSION, "artifact_id": output.artifact_id, "stage": output.stage,
        "kind": output.kind, "path": output.path, "manifest_path": artifact_manifest_path(output.path),
        "size_bytes": size, "sha256": digest, "counts": {"expected": output.expected_records, "observed": observed},
        "provenance": thaw_json(output.provenance), "metadata": thaw_json(output.metadata),
        "created_at": created_at or datetime.now(timezone.utc).isoformat(),
    }
    if entries is not None:
        m["files"] = entries
    validate_json_value(m, "artifact manifest")
    return m


def _load_manifest(path: str) -> Dict[str, Any]:
    mp = artifact_manifest_path(path)
    try:
        value = json.loads(read_stable_regular_file(mp))
    except (OSError, ValueError) as exc:
        raise ValueError(f"artifact ready manifest is unavailable: {mp}") from exc
    if not isinstance(value, dict):
        raise ValueError(f"artifact ready manifest must be an object: {mp}")
    return value


def validate_artifact(output: DeclaredOutput, *, manifest: Mapping[str, Any] | None = None) -> Dict[str, Any]:
    """Check the manifest against the declaration and the bytes on disk; return the manifest."""

    m = dict(manifest if manifest is not None else _load_manifest(output.path))
    required = _MANIFEST_KEYS | ({"files"} if output.kind == "directory" else set())
    if set(m) != required:
        raise ValueError("invalid artifact manifest schema")
    if m["v"] != ARTIFACT_MANIFEST_VERSION:
        raise ValueError("unsupported artifact manifest version")
    if (m["artifact_id"], m["kind"], m["stage"], m["path"]) != (output.artifact_id, output.kind, output.stage,
                                                                 output.path):
        raise ValueError("artifact declaration does not match manifest")
    if m["manifest_path"] != artifact_manifest_path(output.path):
        raise ValueError("artifact manifest path does not match")
    counts = m["counts"]
    if not isinstance(counts, Mapping) or set(counts) != {"expected", "observed"}:
        raise ValueError("invalid artifact counts")
    if counts["expected"] != output.expected_records:
        raise ValueError("artifact expected record count does not match declaration")
    if output.expected_records is not None and counts["observed"] != output.expected_records:
        raise ValueError("artifact observed record count does not match")
    if m["provenance"] != thaw_json(output.provenance) or m["metadata"] != thaw_json(output.metadata):
        raise ValueError("artifact provenance or metadata does not match declaration")
    size, digest, entries = _digest(output.kind, Path(output.path))
    if (m["size_bytes"], m["sha256"]) != (size, digest) or (entries is not None and m["files"] != entries):
        raise ValueError("artifact bytes do not match the ready manifest")
    return m


def publish_artifact(output: DeclaredOutput, *, observed_records: int | None = None) -> Dict[str, Any]:
    """Hash the finished output and write its ready manifest once; re-publication must agree."""

    m = build_artifact_manifest(output, observed_records=observed_records)
    mp = artifact_manifest_path(output.path)
    if os.path.lexists(mp):
        existing = _load_manifest(output.path)
        validate_artifact(output, manifest=existing)
        return existing
    payload = (json.dumps(m, indent=2, sort_keys=True) + "\n").encode()
    if not write_immutable_file(mp, payload):
        existing = _load_manifest(output.path)
        validate_artifact(output, manifest=existing)
        return existing
    return m


def artifact_publication(manifest: Mapping[str, Any]) -> Dict[str, Any]:
    """The identity fields a coordinator compares (same keys as a checkpoint publication)."""

    return {"v": manifest["v"], "artifact_id": manifest["artifact_id"], "path": manifest["path"],
            "size_bytes": manifest["size_bytes"], "sha256": manifest["sha256"],
            "manifest_path": manifest["manifest_path"]}
