"""Execution environment profiles: the strict, site-neutral part of a launch.

(reference: koochak/jobs/profile.py:138-312)

A profile is a small YAML document (version 1):

    version: 1
    id: b200-node
    python: /opt/venv/bin/python3
    environment:
      set: {PATH: /opt/venv/bin:/usr/bin:/bin, CC: /usr/bin/gcc, ...}
      secrets: [WANDB_API_KEY]            # names passed through, never recorded
      create_directories: ["{run_dir}/tmp"]
    requirements:
      executables: [/usr/local/cuda/bin/nvcc]
      files: ["{cwd}/data/index.json"]
      packages: {torch: "2.11.0", numpy: "*"}
    preflight: [c_compiler, cuda, nvcc_sm100a]

Rules: names are environment identifiers; ``PATH`` is explicit and absolute;
variables owned by the scheduler or host (``RUNTIME_ENVIRONMENT``) cannot be
set or declared secret; ``{cwd}`` and ``{run_dir}`` are the only
placeholders; no ``${...}`` interpolation. ``resolve`` fills the placeholders
for one run and returns the record embedded in its launch manifest. The
profile's identity is the SHA-256 of its canonical JSON.

Preflights (run by the runner before the target starts): ``c_compiler``
(needs ``CC``), ``cuda`` (a CUDA device is visible), ``torch_compile`` (needs
``CC`` and ``CXX``), and ``nvcc_sm100a`` (the CUDA compiler accepts
``-gencode arch=compute_100a,code=sm_100a``).
"""

from __future__ import annotations

import hashlib
import json
import re
from dataclasses import dataclass, field
from pathlib import Path, PurePosixPath
from string import Formatter
from types import MappingProxyType
from typing import Any, Dict, Mapping, Tuple

__all__ = ["EnvironmentProfile", "ResolvedEnvironment", "load_environment_profile", "PREFLIGHTS",
           "RUNTIME_ENVIRONMENT"]

_NAME = re.compile(r"[A-Za-z_][A-Za-z0-9_]*\Z")
_PROFILE_ID = re.compile(r"[A-Za-z0-9][A-Za-z0-9_.-]{0,127}\Z")
_PACKAGE = re.compile(r"[A-Za-z_][A-Za-z0-9_.-]*\Z")
_PLACEHOLDERS = {"cwd", "run_dir"}
PREFLIGHTS = frozenset({"c_compiler", "cuda", "torch_compile", "nvcc_sm100a"})
# Owned by the scheduler or the host; the runner always passes them through.
RUNTIME_ENVIRONMENT: Tuple[str, ...] = (
    "HOME", "USER", "LOGNAME", "LANG", "LC_*", "TMPDIR", "XDG_RUNTIME_DIR", "SLURM_*", "SCRUFFY_*",
    "CUDA_VISIBLE_DEVICES", "RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
)


def canonical_sha256(value: object) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def _matches(name: str, pattern: str) -> bool:
    return name.startswith(pattern[:-1]) if pattern.endswith("*") else name == pattern


def _runtime_owned(name: str) -> bool:
    return any(_matches(name, p) for p in RUNTIME_ENVIRONMENT)


def _abs(value: object, what: str) -> str:
    if not isinstance(value, str) or "\x00" in value or not PurePosixPath(value).is_absolute():
        raise ValueError(f"{what} must be an absolute POSIX path")
    return value


def _fill(value: str, variables: Mapping[str, str], what: str) -> str:
    used = {f for _, f, _, _ in Formatter().parse(value) if f is not None}
    if used - _PLACEHOLDERS:
        raise ValueError(f"{what} contains unsupported placeholders: {sorted(used - _PLACEHOLDERS)!r}")
    return value.format_map(variables)


@dataclass(frozen=True)
class ResolvedEnvironment:
    profile_id: str
    profile_sha256: str
    python: str
    variables: Mapping[str, str]
    preserve: Tuple[str, ...]
    secrets: Tuple[str, ...]
    create_directories: Tuple[str, ...]
    executables: Tuple[str, ...]
    files: Tuple[str, ...]
    packages: Mapping[str, str]
    preflight: Tuple[str, ...]

    def to_dict(self) -> Dict[str, Any]:
        return {
            "id": self.profile_id, "sha256": self.profile_sha256, "python": self.python,
            "environment": {"set": dict(self.variables), "preserve": list(self.preserve),
                            "secrets": list(self.secrets), "create_directories": list(self.create_directories)},
            "requirements": {"executables": list(self.executables), "files": list(self.files),
                             "packages": dict(self.packages)},
            "preflight": list(self.preflight),
        }


@dataclass(frozen=True)
class EnvironmentProfile:
    profile_id: str
    python: str
    variables: Mapping[str, str]
    secrets: Tuple[str, ...] = ()
    create_directories: Tuple[str, ...] = ()
    executables: Tuple[str, ...] = ()
    files: Tuple[str, ...] = ()
    packages: Mapping[str, str] = field(default_factory=lambda: MappingProxyType({}))
    preflight: Tuple[str, ...] = ()

    def __post_init__(self) -> None:
        if not isinstance(self.profile_id, str) or not _PROFILE_ID.fullmatch(self.profile_id):
            raise ValueError("profile id must contain only letters, digits, '.', '_' or '-'")
        _abs(self.python, "python")
        env = dict(self.variables)
        for k, v in env.items():
            if not (isinstance(k, str) and _NAME.fullmatch(k) and isinstance(v, str) and "\x00" not in v):
                raise ValueError("environment.set must map valid names to strings without NUL bytes")
            if _runtime_owned(k):
                raise ValueError(f"environment.set cannot override runtime-owned {k}")
        if "PATH" not in env:
            raise ValueError("environment.set must define an explicit PATH")
        if any(not part.startswith("/") for part in env["PATH"].split(":")):
            raise ValueError("PATH must contain only non-empty absolute entries")
        secrets = tuple(self.secrets)
        for name in secrets:
            if not isinstance(name, str) or not _NAME.fullmatch(name):
                raise ValueError("environment.secrets entries must be exact names")
            if name in env:
                raise ValueError("secret values cannot also appear in environment.set")
            if _runtime_owned(name):
                raise ValueError("secrets cannot override runtime-owned environment names")
        execs = tuple(_abs(x, "requirements.executables") for x in self.executables)
        pk = dict(self.packages)
        if not all(isinstance(n, str) and _PACKAGE.fullmatch(n) and isinstance(v, str) and v for n, v in pk.items()):
            raise ValueError("requirements.packages must map import names to versions or '*'")
        bad = [c for c in self.preflight if c not in PREFLIGHTS]
        if bad:
            raise ValueError(f"preflight entries must be chosen from {sorted(PREFLIGHTS)!r}")
        if "c_compiler" in self.preflight and "CC" not in env:
            raise ValueError("c_compiler preflight requires an explicit CC")
        if "torch_compile" in self.preflight and not {"CC", "CXX"} <= env.keys():
            raise ValueError("torch_compile preflight requires explicit CC and CXX")
        for k in {"CC", "CXX"} & env.keys():
            _abs(env[k], f"environment.set.{k}")
        for p in (*self.create_directories, *self.files):
            _abs(_fill(p, {"cwd": "/cwd", "run_dir": "/run"}, "profile path"), "profile path")
        object.__setattr__(self, "variables", MappingProxyType(dict(sorted(env.items()))))
        object.__setattr__(self, "secrets", secrets)
        object.__setattr__(self, "create_directories", tuple(self.create_directories))
        object.__setattr__(self, "executables", execs)
        object.__setattr__(self, "files", tuple(self.files))
        object.__setattr__(self, "packages", MappingProxyType(dict(sorted(pk.items()))))
        object.__setattr__(self, "preflight", tuple(self.preflight))

    def to_dict(self) -> Dict[str, Any]:
        return {
            "version": 1, "id": self.profile_id, "python": self.python,
            "environment": {"set": dict(self.variables), "secrets": list(self.secrets),
                            "create_directories": list(self.create_directories)},
            "requirements": {"executables": list(self.executables), "files": list(self.files),
                             "packages": dict(self.packages)},
            "preflight": list(self.preflight),
        }

    @property
    def sha256(self) -> str:
        return canonical_sha256(self.to_dict())

    def resolve(self, *, cwd: str, run_dir: str) -> ResolvedEnvironment:
        vals = {"cwd": _abs(cwd, "cwd"), "run_dir": _abs(run_dir, "run_dir")}
        return ResolvedEnvironment(
            profile_id=self.profile_id, profile_sha256=self.sha256, python=self.python,
            variables=MappingProxyType({k: _fill(v, vals, f"environment.set.{k}") for k, v in self.variables.items()}),
            preserve=RUNTIME_ENVIRONMENT, secrets=self.secrets,
            create_directories=tuple(_abs(_fill(v, vals, "environment.create_directories"), "directory")
                                     for v in self.create_directories),
            executables=self.executables,
            files=tuple(_abs(_fill(v, vals, "requirements.files"), "file") for v in self.files),
            packages=self.packages, preflight=self.preflight,
        )


def _section(doc: Mapping[str, Any], key: str, allowed: set, what: str) -> Dict[str, Any]:
    v = doc.get(key, {}) or {}
    if not isinstance(v, Mapping) or not all(isinstance(k, str) for k in v):
        raise ValueError(f"{what} must be a mapping with string keys")
    extra = set(v) - allowed
    if extra:
        raise ValueError(f"invalid {what}: unexpected {sorted(extra)!r}")
    return dict(v)


def _str_list(v: object, what: str) -> Tuple[str, ...]:
    if not isinstance(v, (list, tuple)) or not all(isinstance(x, str) and x for x in v):
        raise ValueError(f"{what} must be a list of non-empty strings")
    return tuple(v)


def load_environment_profile(source: str | Path) -> EnvironmentProfile:
    """Load one strict YAML profile (no interpolation, no unknown keys)."""

    import yaml

    text = Path(source).read_text()
    if "${" in text:
        raise ValueError("environment profiles do not permit interpolation")
    doc = yaml.safe_load(text)
    if not isinstance(doc, Mapping) or not all(isinstance(k, str) for k in doc):
        raise ValueError("profile must be a mapping with string keys")
    missing = {"version", "id", "python"} - set(doc)
    extra = set(doc) - {"version", "id", "python", "environment", "requirements", "preflight"}
    if missing or extra:
        raise ValueError(f"invalid profile: missing {sorted(missing)!r}, unexpected {sorted(extra)!r}")
    if doc["version"] != 1:
        raise ValueError("profile version must be 1")
    env = _section(doc, "environment", {"set", "secrets", "create_directories"}, "environment")
    req = _section(doc, "requirements", {"executables", "files", "packages"}, "requirements")
    variables = env.get("set", {}) or {}
    packages = req.get("packages", {}) or {}
    if not isinstance(variables, Mapping) or not isinstance(packages, Mapping):
        raise ValueError("environment.set and requirements.packages must be mappings")
    return EnvironmentProfile(
        profile_id=doc["id"], python=doc["python"], variables=dict(variables),
        secrets=_str_list(env.get("secrets", []), "environment.secrets"),
        create_directories=_str_list(env.get("create_directories", []), "environment.create_directories"),
        executables=_str_list(req.get("executables", []), "requirements.executables"),
        files=_str_list(req.get("files", []), "requirements.files"),
        packages={str(k): str(v) for k, v in packages.items()},
        preflight=_str_list(doc.get("preflight", []), "preflight"),
    )
