"""Compile an experiment (config + patches + environment profile) into one launch.

(reference: koochak/jobs/manifest.py:79-348)

``prepare_run`` produces a ``PreparedRun``: three immutable artifacts under
``run_dir`` and the argv that starts them.

* ``config.yaml``   the resolved training config (``train.out_dir`` set to the
                    run directory, then every ``ConfigPatch`` applied);
* ``koochak-runtime.zip``  every ``.py`` file of this package, zipped with
                    fixed timestamps (so the same source gives the same
                    digest), for the runner to import;
* ``launch.json``   the manifest: argv, cwd, the resolved environment
                    profile, declared outputs, preemption policy and the
                    digests of the other two files.

``runner_argv()`` is ``python -I -c <bootstrap> runtime sha manifest sha``:
the bootstrap checks both digests before importing anything from the zip,
then runs ``koochak_b200.jobs.runner``. Nothing here imports PyTorch.

``Preemptible`` marks a run that a scheduler may evacuate (SIGUSR1) and
resubmit: it adds ``<section>.evacuation_enabled: true`` and
``<section>.resume: auto`` to the config, and its ``recovery()`` policy
(retry on allocation replacement or evacuation, up to ``max_attempts``).
"""

from __future__ import annotations

import hashlib
import io
import json
import posixpath
import re
import zipfile
from dataclasses import dataclass
from pathlib import Path, PurePosixPath
from typing import Any, Dict, List, Optional, Sequence, Tuple

from ..storage.artifact import DeclaredOutput
from ..storage.immutable import write_immutable_file
from .profile import EnvironmentProfile

__all__ = ["ConfigPatch", "Preemptible", "PreparedRun", "Artifact", "materialize_config", "prepare_run", "stage_run",
           "PREEMPTIBLE_RETRY_ON", "RUNTIME_NAME"]

_JOB_NAME = re.compile(r"[A-Za-z0-9][A-Za-z0-9_.-]{0,127}\Z")
RUNTIME_NAME = "koochak-runtime.zip"
PREEMPTIBLE_RETRY_ON = ("allocation_replaced", "allocation_incarnation_changed", "evacuated")

# Runs under `python -I -c`: standard library only, digests verified before import.
BOOTSTRAP = """\
import hashlib, json, runpy, sys
from pathlib import Path
rt_path, rt_sha, man_path, man_sha = sys.argv[1:5]
man = Path(man_path).read_bytes()
if hashlib.sha256(man).hexdigest() != man_sha:
    raise SystemExit("launch manifest digest differs")
rt = json.loads(man).get("runner_runtime")
if not isinstance(rt, dict) or rt.get("path") != rt_path or rt.get("sha256") != rt_sha:
    raise SystemExit("runner runtime does not match its launch manifest")
if hashlib.sha256(Path(rt_path).read_bytes()).hexdigest() != rt_sha:
    raise SystemExit("runner runtime digest differs")
sys.path.insert(0, rt_path)
sys.argv = ["koochak_b200.jobs.runner", man_path, man_sha]
runpy.run_module("koochak_b200.jobs.runner", run_name="__main__")
"""


def _sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def runtime_package() -> bytes:
    """Deterministic zip of this package's Python sources."""

    root = Path(__file__).resolve().parents[1]
    buf = io.BytesIO()
    with zipfile.ZipFile(buf, "w", compression=zipfile.ZIP_DEFLATED) as zf:
        for src in sorted(root.rglob("*.py")):
            rel = src.relative_to(root)
            if "_build" in rel.parts or "__pycache__" in rel.parts:
                continue
            info = zipfile.ZipInfo(f"{root.name}/{rel.as_posix()}", date_time=(1980, 1, 1, 0, 0, 0))
            info.compress_type = zipfile.ZIP_DEFLATED
            info.external_attr = 0o644 << 16
            zf.writestr(info, src.read_bytes())
    return buf.getvalue()


def _abs(value: object, what: str) -> str:
    if not isinstance(value, str) or "\x00" in value or not PurePosixPath(value).is_absolute():
        raise ValueError(f"{what} must be an absolute POSIX path")
    return value


@dataclass(frozen=True)
class ConfigPatch:
    """A dotted-path update applied to the config before the launch is prepared."""

    path: str
    value: Any
    merge: bool = True

    def __post_init__(self) -> None:
        if not isinstance(self.path, str) or not self.path.strip():
            raise ValueError("patch path must be non-empty")


@dataclass(frozen=True)
class Preemptible:
    grace_seconds: int = 600
    max_attempts: int = 10
    config_section: Optional[str] = "train"

    def __post_init__(self) -> None:
        if type(self.grace_seconds) is not int or self.grace_seconds < 1:
            raise ValueError("grace_seconds must be a positive integer")
        if type(self.max_attempts) is not int or not 2 <= self.max_attempts <= 10:
            raise ValueError("max_attempts must be an integer from 2 through 10")
        if self.config_section is not None and (not isinstance(self.config_section, str)
                                                or not self.config_section.strip()):
            raise ValueError("config_section must be a non-empty string or None")

    def recovery(self) -> Dict[str, Any]:
        return {"max_attempts": self.max_attempts, "retry_on": list(PREEMPTIBLE_RETRY_ON),
                "evacuation": {"signal": "USR1", "grace_seconds": self.grace_seconds}}

    def config_patches(self, patches: Sequence[ConfigPatch]) -> Tuple[ConfigPatch, ...]:
        if self.config_section is None:
            return ()
        need = {f"{self.config_section}.evacuation_enabled": True, f"{self.config_section}.resume": "auto"}
        for p in patches:
            if p.path in need and p.value != need[p.path]:
                raise ValueError(f"patch {p.path}={p.value!r} conflicts with preemptible; "
                                 f"preemptible runs require {need[p.path]!r}")
        return tuple(ConfigPatch(k, v) for k, v in need.items())


def _preemption(value) -> Optional[Preemptible]:
    if isinstance(value, Preemptible):
        return value
    if type(value) is bool:
        return Preemptible() if value else None
    raise TypeError("preemptible must be a bool or a Preemptible")


@dataclass(frozen=True)
class Artifact:
    path: str
    content: bytes
    sha256: str


@dataclass(frozen=True)
class PreparedRun:
    name: str
    cwd: str
    run_dir: str
    python: str
    manifest_path: str
    manifest_sha256: str
    artifacts: Tuple[Artifact, ...]
    declared_outputs: Tuple[DeclaredOutput, ...] = ()
    preemption: Optional[Preemptible] = None

    def runner_argv(self) -> List[str]:
        rt_path = posixpath.join(self.run_dir, RUNTIME_NAME)
        rt = next(a for a in self.artifacts if a.path == rt_path)
        return [self.python, "-I", "-c", BOOTSTRAP, rt_path, rt.sha256, self.manifest_path, self.manifest_sha256]


def _set_dotted(cfg: Dict[str, Any], dotted: str, value: Any, merge: bool) -> None:
    keys = dotted.split(".")
    node = cfg
    for k in keys[:-1]:
        nxt = node.get(k)
        if not isinstance(nxt, dict):
            nxt = {}
            node[k] = nxt
        node = nxt
    last = keys[-1]
    if merge and isinstance(node.get(last), dict) and isinstance(value, dict):
        merged = dict(node[last])
        merged.update(value)
        node[last] = merged
    else:
        node[last] = value


def materialize_config(base_config: str | Path, *, run_dir: str, patches: Sequence[ConfigPatch] = (),
                       out_dir_config_key: Optional[str] = "train.out_dir") -> str:
    """The final YAML text of a run's config (``${a.b}`` references resolved)."""

    import yaml

    from ..config import resolve

    doc = yaml.safe_load(Path(base_config).read_text()) or {}
    if not isinstance(doc, dict):
        raise ValueError("config must be a mapping")
    if out_dir_config_key:
        _set_dotted(doc, out_dir_config_key, run_dir, True)
    for p in patches:
        _set_dotted(doc, p.path, p.value, p.merge)
    resolved = resolve(doc)
    from ..config import to_container

    return yaml.safe_dump(to_container(resolved), sort_keys=False)


def _resolve_args(args: Sequence[str], *, cwd: str, run_dir: str, config_path: Optional[str]) -> List[str]:
    if isinstance(args, (str, bytes)) or not args:
        raise ValueError("python_args must contain at least one argument")
    subs = {"{cwd}": cwd, "{run_dir}": run_dir}
    if config_path is not None:
        subs["{config}"] = config_path
    out = []
    for a in args:
        if not isinstance(a, str) or not a or "\x00" in a:
            raise ValueError("python_args must contain non-empty strings without NUL bytes")
        for k, v in subs.items():
            a = a.replace(k, v)
        if "{config}" in a:
            raise ValueError("{config} requires base_config")
        out.append(a)
    return out


def prepare_run(*, name: str, profile: EnvironmentProfile, python_args: Sequence[str], cwd: str, run_dir: str,
                base_config: str | Path | None = None, patches: Sequence[ConfigPatch] = (),
                out_dir_config_key: Optional[str] = "train.out_dir",
                declared_outputs: Sequence[DeclaredOutput] = (), preemptible: bool | Preemptible = False
                ) -> PreparedRun:
    """Build the launch in memory (no I/O besides reading the base config and sources)."""

    if not isinstance(name, str) or not _JOB_NAME.fullmatch(name):
        raise ValueError("name must contain only letters, digits, '.', '_' or '-'")
    pre = _preemption(preemptible)
    patches = tuple(patches)
    if pre is not None and pre.config_section is not None:
        if base_config is None:
            raise ValueError("preemptible runs need base_config to enable evacuation and auto-resume; "
                             "use Preemptible(config_section=None) if the entrypoint enables both itself")
        patches = patches + pre.config_patches(patches)
    cwd = _abs(cwd, "cwd")
    run_dir = _abs(run_dir, "run_dir").rstrip("/") or "/"
    manifest_path = posixpath.join(run_dir, "launch.json")
    config_path = posixpath.join(run_dir, "config.yaml") if base_config is not None else None
    env = profile.resolve(cwd=cwd, run_dir=run_dir)
    outputs = tuple(declared_outputs)
    ids = [o.artifact_id for o in outputs]
    if len(set(ids)) != len(ids):
        raise ValueError("declared outputs must have unique artifact IDs")
    doc: Dict[str, Any] = {
        "v": 1, "name": name, "cwd": cwd, "run_dir": run_dir,
        "argv": [env.python, *_resolve_args(python_args, cwd=cwd, run_dir=run_dir, config_path=config_path)],
        "environment": env.to_dict(), "preflight_result_path": posixpath.join(run_dir, "preflight.json"),
        "outputs": [o.to_dict() for o in outputs],
    }
    if pre is not None:
        doc["preemption"] = pre.recovery()
    arts: List[Artifact] = []
    if base_config is not None and config_path is not None:
        text = materialize_config(base_config, run_dir=run_dir, patches=patches,
                                  out_dir_config_key=out_dir_config_key).encode()
        doc["config"] = {"path": config_path, "sha256": _sha(text)}
        arts.append(Artifact(config_path, text, _sha(text)))
    rt_path = posixpath.join(run_dir, RUNTIME_NAME)
    rt = runtime_package()
    doc["runner_runtime"] = {"path": rt_path, "sha256": _sha(rt)}
    arts.append(Artifact(rt_path, rt, _sha(rt)))
    man = (json.dumps(doc, indent=2, sort_keys=True, ensure_ascii=False) + "\n").encode()
    arts.append(Artifact(manifest_path, man, _sha(man)))
    return PreparedRun(name=name, cwd=cwd, run_dir=run_dir, python=env.python, manifest_path=manifest_path,
                       manifest_sha256=_sha(man), artifacts=tuple(arts), declared_outputs=outputs, preemption=pre)


def stage_run(prepared: PreparedRun) -> None:
    """Write the prepared artifacts (immutably) on a directly mounted filesystem."""

    for a in prepared.artifacts:
        write_immutable_file(a.path, a.content)
