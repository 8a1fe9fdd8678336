"""Isolated launcher: verify a prepared launch, check the environment, run it.

(reference: koochak/jobs/runner.py:53-707)

    python -I -c <bootstrap> runtime.zip <sha> launch.json <sha>   (from PreparedRun.runner_argv)
    python -m koochak_b200.jobs.runner launch.json <sha>

Order of work:

1. the manifest digest must match; the environment is rebuilt from scratch:
   the profile's ``set`` values, then the scheduler-owned names it preserves,
   then the declared secrets (which must be present);
2. declared directories are created, the config digest is checked, required
   executables / files / packages (with versions) are observed, and the
   profile's preflights run (``c_compiler``, ``cuda``, ``torch_compile``,
   ``nvcc_sm100a``); the outcome goes to ``preflight.json`` either way and a
   failure exits 78;
3. the workload runs as its own process group. SIGUSR1 to the runner is
   recorded, never acted on inside the handler; for a preemptible run the
   runner creates ``requested`` in a private directory named by
   ``KOOCHAK_EVACUATION_DIR`` and every rank sees it at its next update.
   Once the workload writes ``evacuated`` the run reports exit 75 whatever
   its launcher returns; a leader that lingers gets SIGTERM after 10 s and
   SIGKILL 30 s later. Descendants left behind by a finished leader are
   cleaned and reported;
4. declared outputs must have valid ready manifests; inside a Scruffy worker
   each is announced as a ``workload.artifact`` event.
"""

from __future__ import annotations

import hashlib
import importlib
import json
import os
import signal
import subprocess
import sys
import tempfile
import time
from datetime import datetime, timezone
from pathlib import Path
from typing import Any, Dict, List, Mapping, Optional, Tuple

from ..interruption import EVACUATED_FILE, EVACUATION_DIR_ENV, EVACUATION_EXIT_CODE, EVACUATION_REQUEST_FILE
from ..storage.artifact import DeclaredOutput, artifact_publication, validate_artifact

__all__ = ["PreflightError", "build_environment", "execute_manifest", "main", "PREFLIGHT_EXIT_CODE"]

PREFLIGHT_EXIT_CODE = 78
EXIT_GRACE_S = 10.0
KILL_GRACE_S = 30.0
MARKER_WAIT_S = 0.5

_CHILD_BOOTSTRAP = """\
import hashlib, runpy, sys
from pathlib import Path
rt_path, rt_sha, roots = sys.argv[1:4]
if hashlib.sha256(Path(rt_path).read_bytes()).hexdigest() != rt_sha:
    raise SystemExit("runner runtime digest differs")
sys.path.insert(0, rt_path)
sys.argv = ["koochak_b200.jobs.isolated_exec", roots, "--", *sys.argv[5:]]
runpy.run_module("koochak_b200.jobs.isolated_exec", run_name="__main__")
"""


class PreflightError(RuntimeError):
    pass


def _canon_sha(value: object) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def _matches(name: str, pattern: str) -> bool:
    return name.startswith(pattern[:-1]) if pattern.endswith("*") else name == pattern


def build_environment(environment: Mapping[str, Any], source: Mapping[str, str]) -> Dict[str, str]:
    s = environment["environment"]
    out = dict(s["set"])
    out.update({k: v for k, v in source.items() if any(_matches(k, p) for p in s["preserve"])})
    missing = [n for n in s["secrets"] if n not in source]
    if missing:
        raise PreflightError(f"missing secret environment names: {missing!r}")
    out.update({n: source[n] for n in s["secrets"]})
    return out


def _load_manifest(path: str, sha: str) -> Dict[str, Any]:
    raw = Path(path).read_bytes()
    got = hashlib.sha256(raw).hexdigest()
    if got != sha:
        raise PreflightError(f"launch manifest digest differs: expected {sha}, got {got}")
    doc = json.loads(raw)
    if not isinstance(doc, dict) or doc.get("v") != 1:
        raise PreflightError("launch manifest must be a version-1 object")
    return doc


def _need_exec(path: str) -> None:
    if not Path(path).is_file() or not os.access(path, os.X_OK):
        raise PreflightError(f"required executable is unavailable: {path}")


def _import_roots(environment: Mapping[str, Any]) -> Tuple[str, ...]:
    pp = environment["environment"]["set"].get("PYTHONPATH", "")
    if not isinstance(pp, str):
        raise PreflightError("environment.set.PYTHONPATH must be a string")
    return tuple(x for x in pp.split(os.pathsep) if x)


def _observe_requirements(environment: Mapping[str, Any]) -> Dict[str, str]:
    req = environment["requirements"]
    seen: Dict[str, str] = {}
    _need_exec(environment["python"])
    if Path(sys.executable).resolve() != Path(environment["python"]).resolve():
        raise PreflightError(f"runner interpreter differs: expected {environment['python']}, got {sys.executable}")
    for exe in req["executables"]:
        _need_exec(exe)
        seen[f"executable:{exe}"] = "available"
    for f in req["files"]:
        if not Path(f).is_file():
            raise PreflightError(f"required file is unavailable: {f}")
        seen[f"file:{f}"] = "available"
    for root in reversed(_import_roots(environment)):
        if root not in sys.path:
            sys.path.insert(0, root)
    for mod_name, want in req["packages"].items():
        try:
            mod = importlib.import_module(mod_name)
        except ModuleNotFoundError as exc:
            if exc.name in (mod_name, mod_name.split(".", 1)[0]):
                raise PreflightError(f"required package is not importable: {mod_name}") from exc
            raise PreflightError(f"required package is missing a dependency: {mod_name}: {exc.name}") from exc
        except ImportError as exc:
            raise PreflightError(f"required package is incompatible: {mod_name}: {exc}") from exc
        have = str(getattr(mod, "__version__", "unknown"))
        if want != "*" and have != want:
            raise PreflightError(f"{mod_name} version differs: expected {want}, got {have}")
        seen[f"package:{mod_name}"] = have
    return seen


def _run(cmd: List[str], timeout: float = 180) -> None:
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, check=False)
    except (OSError, subprocess.TimeoutExpired) as exc:
        raise PreflightError(f"preflight command could not run: {cmd[0]}: {exc}") from exc
    if r.returncode:
        raise PreflightError(f"preflight command failed ({r.returncode}): {cmd[0]}: "
                             f"{(r.stderr or r.stdout)[-4000:].strip()}")


def _pf_c_compiler() -> None:
    cc = os.environ.get("CC", "")
    _need_exec(cc)
    with tempfile.TemporaryDirectory(prefix="kb-cc-") as d:
        (Path(d) / "p.c").write_text("int main(void) { return 0; }\n")
        _run([cc, str(Path(d) / "p.c"), "-o", str(Path(d) / "p")], timeout=30)


def _pf_cuda() -> None:
    code = ("import torch\nassert torch.cuda.is_available() and torch.cuda.device_count() >= 1\n"
            "x = torch.zeros(1, device='cuda'); torch.cuda.synchronize(); assert float(x.item()) == 0.0\n")
    _run([sys.executable, "-I", "-c", code])


def _pf_torch_compile() -> None:
    code = ("import torch\n@torch.compile(fullgraph=True)\ndef f(v):\n    return v + 1\n"
            "r = f(torch.zeros(1, device='cuda')); torch.cuda.synchronize(); assert r.item() == 1\n")
    _run([sys.executable, "-I", "-c", code])


def _pf_nvcc_sm100a() -> None:
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    _need_exec(nvcc)
    with tempfile.TemporaryDirectory(prefix="kb-nvcc-") as d:
        src = Path(d) / "p.cu"
        src.write_text("__global__ void k(int* p) { if (p) *p = 1; }\n")
        _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-c", str(src), "-o", str(Path(d) / "p.o")],
             timeout=120)


PREFLIGHT_CHECKS = {"c_compiler": _pf_c_compiler, "cuda": _pf_cuda, "torch_compile": _pf_torch_compile,
                    "nvcc_sm100a": _pf_nvcc_sm100a}


def _write_result(path: str, doc: Mapping[str, Any]) -> None:
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=f".{target.name}.", dir=target.parent)
    try:
        with os.fdopen(fd, "w") as fh:
            json.dump(doc, fh, indent=2, sort_keys=True)
            fh.write("\n")
            fh.flush()
            os.fsync(fh.fileno())
        os.chmod(tmp, 0o444)
        os.replace(tmp, target)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)


def _outputs(doc: Mapping[str, Any]) -> Tuple[DeclaredOutput, ...]:
    raw = doc.get("outputs", [])
    if not isinstance(raw, list):
        raise PreflightError("launch manifest outputs must be a JSON array")
    try:
        outs = tuple(DeclaredOutput.from_dict(v) for v in raw)
    except (TypeError, ValueError) as exc:
        raise PreflightError(f"invalid declared output: {exc}") from exc
    if len({o.artifact_id for o in outs}) != len(outs):
        raise PreflightError("launch manifest outputs must have unique artifact IDs")
    return outs


def _note(kind: str, **fields: Any) -> None:
    print(json.dumps({"kind": kind, **fields}, sort_keys=True), file=sys.stderr, flush=True)


class EvacuationRelay:
    """Records SIGUSR1 for the runner's life; after an evacuation, SIGTERM exits 75."""

    def __init__(self) -> None:
        self.requested = False
        self.evacuated = False
        self._prev_usr1: Any = signal.SIG_DFL
        self._prev_term: Any = None
        self._control: Optional[Path] = None
        self._group: Optional[int] = None

    def __enter__(self) -> "EvacuationRelay":
        self._prev_usr1 = signal.getsignal(signal.SIGUSR1)
        signal.signal(signal.SIGUSR1, self._on_usr1)
        return self

    def __exit__(self, *exc: object) -> None:
        if self._prev_term is not None:
            signal.signal(signal.SIGTERM, self._prev_term)
            self._prev_term = None
        signal.signal(signal.SIGUSR1, self._prev_usr1)

    def _on_usr1(self, signum, frame) -> None:
        self.requested = True

    def watch(self, control: Path, group: int) -> None:
        self._control, self._group = control, group
        if self._prev_term is None:
            prev = signal.getsignal(signal.SIGTERM)
            self._prev_term = signal.SIG_DFL if prev is None else prev
            signal.signal(signal.SIGTERM, self._on_term)

    def release(self, *, evacuated: bool) -> None:
        self.evacuated = self.evacuated or evacuated
        self._control = self._group = None

    def _done(self) -> bool:
        return self.evacuated or (self._control is not None and (self._control / EVACUATED_FILE).exists())

    def _on_term(self, signum, frame) -> None:
        deadline = time.monotonic() + MARKER_WAIT_S
        while not self._done() and time.monotonic() < deadline:
            time.sleep(0.02)
        if self._done():
            if self._group is not None:
                try:
                    os.killpg(self._group, signal.SIGKILL)
                except ProcessLookupError:
                    pass
            os.write(2, b'{"kind": "evacuated_runner_terminated"}\n')
            os._exit(EVACUATION_EXIT_CODE)
        prev, self._prev_term = self._prev_term, None
        signal.signal(signal.SIGTERM, prev)
        if callable(prev):
            prev(signum, frame)
        elif prev == signal.SIG_DFL:
            os.kill(os.getpid(), signum)


def _child_argv(argv: List[str], roots: Tuple[str, ...], rt_path: Optional[str], rt_sha: Optional[str]) -> List[str]:
    """Route an isolated (``-I``) Python child through the import-root bootstrap."""

    if not roots or not rt_path or not rt_sha or not Path(argv[0]).name.startswith("python") or "-I" not in argv[1:]:
        return argv
    rest = [a for a in argv[1:] if a != "-I"]
    return [argv[0], "-I", "-c", _CHILD_BOOTSTRAP, rt_path, rt_sha, json.dumps(list(roots), separators=(",", ":")),
            "--", *rest]


def _group_alive(pg: int) -> bool:
    try:
        os.killpg(pg, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    return True


def _quiesce(pg: int, *, stopped: bool, wait_s: float = 1.0) -> None:
    if not _group_alive(pg):
        return
    for sig in (signal.SIGTERM, signal.SIGKILL):
        try:
            os.killpg(pg, sig)
        except ProcessLookupError:
            break
        end = time.monotonic() + wait_s
        while _group_alive(pg) and time.monotonic() < end:
            time.sleep(0.01)
        if not _group_alive(pg):
            break
    if _group_alive(pg):
        raise PreflightError("managed workload process group could not be quiesced")
    if not stopped:
        raise PreflightError("managed workload left background descendants")


def run_managed_child(argv: List[str], *, cwd: str, environment: Mapping[str, str], relay: EvacuationRelay,
                      preemptible: bool, import_roots: Tuple[str, ...] = (), runtime_path: Optional[str] = None,
                      runtime_sha256: Optional[str] = None, poll_s: float = 0.1) -> int:
    if relay.requested and preemptible:
        return EVACUATION_EXIT_CODE
    with tempfile.TemporaryDirectory(prefix="kb-evacuation-") as tmp:
        control = Path(tmp)
        env = dict(environment)
        if preemptible:
            env[EVACUATION_DIR_ENV] = tmp
        forwarded = noted = False
        evacuated_at: Optional[float] = None
        stops: List[Tuple[float, signal.Signals]] = []
        try:
            child = subprocess.Popen(_child_argv(argv, import_roots, runtime_path, runtime_sha256), cwd=cwd,
                                     env=env, start_new_session=True)
            while True:
                try:
                    rc = child.wait(timeout=poll_s)
                    break
                except subprocess.TimeoutExpired:
                    pass
                if relay.requested and not forwarded:
                    if preemptible:
                        relay.watch(control, child.pid)
                        (control / EVACUATION_REQUEST_FILE).touch()
                        _note("evacuation_requested")
                        forwarded = True
                    elif not noted:
                        _note("evacuation_ignored", reason="run_not_preemptible")
                        noted = True
                if not preemptible:
                    continue
                if evacuated_at is None and (control / EVACUATED_FILE).exists():
                    evacuated_at = time.monotonic()
                    stops = [(EXIT_GRACE_S, signal.SIGTERM), (EXIT_GRACE_S + KILL_GRACE_S, signal.SIGKILL)]
                if stops and evacuated_at is not None and time.monotonic() - evacuated_at >= stops[0][0]:
                    _, sig = stops.pop(0)
                    _note("evacuated_leader_stopped", signal=sig.name)
                    try:
                        os.killpg(child.pid, sig)
                    except ProcessLookupError:
                        pass
            evacuated = preemptible and (control / EVACUATED_FILE).exists()
            _quiesce(child.pid, stopped=evacuated_at is not None and len(stops) < 2)
        except OSError as exc:
            raise PreflightError(f"managed workload could not run: {exc}") from exc
        finally:
            relay.release(evacuated=preemptible and (control / EVACUATED_FILE).exists())
    status = 128 + abs(rc) if rc < 0 else rc
    if evacuated and status != EVACUATION_EXIT_CODE:
        _note("evacuation_completed", workload_returncode=status)
        return EVACUATION_EXIT_CODE
    return status


def _publish_outputs(outputs: Tuple[DeclaredOutput, ...], env: Mapping[str, str]) -> None:
    first = [validate_artifact(o) for o in outputs]
    root, job = env.get("SCRUFFY_ROOT"), env.get("SCRUFFY_JOB_ID")
    publish = None
    if "SCRUFFY_ROOT" in env or "SCRUFFY_JOB_ID" in env:
        if not root or not job:
            raise PreflightError("declared outputs require both SCRUFFY_ROOT and SCRUFFY_JOB_ID for Scruffy workers")
        try:
            from scruffy import publish_event as publish  # type: ignore
        except ModuleNotFoundError as exc:
            if exc.name == "scruffy":
                raise PreflightError("declared outputs require the Scruffy client") from exc
            raise PreflightError("the installed Scruffy client is missing a dependency") from exc
        except ImportError as exc:
            raise PreflightError("the installed Scruffy client is incompatible") from exc
    for out, m0 in zip(outputs, first):
        m = validate_artifact(out)
        if m != m0:
            raise PreflightError(f"declared output changed during publication: {out.artifact_id}")
        if publish is None:
            continue
        ident = hashlib.sha256(f"{job}\0{out.artifact_id}\0{m['sha256']}".encode()).hexdigest()
        publish(Path(root), job_id=job, kind="workload.artifact", event_id=f"koochak-artifact-{ident}",
                source={"name": "koochak-runner"},
                data={"artifact_type": out.stage or out.kind, "location": out.path,
                      "publication": artifact_publication(m), "stage": out.stage,
                      "provenance": dict(out.provenance), "counts": dict(m["counts"]),
                      "metadata": dict(out.metadata)})


def _is_preemptible(doc: Mapping[str, Any]) -> bool:
    pol = doc.get("preemption")
    if pol is None:
        return False
    if not isinstance(pol, Mapping) or set(pol) != {"max_attempts", "retry_on", "evacuation"}:
        raise PreflightError("launch manifest preemption must be a recovery policy object")
    return True


def execute_manifest(manifest_path: str, expected_sha256: str) -> int:
    with EvacuationRelay() as relay:
        return _execute(manifest_path, expected_sha256, relay)


def _execute(manifest_path: str, sha: str, relay: EvacuationRelay) -> int:
    doc = _load_manifest(manifest_path, sha)
    env_doc = doc["environment"]
    secrets = set(env_doc["environment"]["secrets"])
    result_path = doc["preflight_result_path"]
    result: Dict[str, Any] = {"v": 1, "manifest_sha256": sha, "profile_id": env_doc["id"],
                              "profile_sha256": env_doc["sha256"],
                              "recorded_at": datetime.now(timezone.utc).isoformat()}
    try:
        preemptible = _is_preemptible(doc)
        clean = build_environment(env_doc, os.environ)
        os.environ.clear()
        os.environ.update(clean)
        for d in env_doc["environment"]["create_directories"]:
            Path(d).mkdir(parents=True, exist_ok=True)
        cfg = doc.get("config")
        if cfg is not None:
            got = hashlib.sha256(Path(cfg["path"]).read_bytes()).hexdigest()
            if got != cfg["sha256"]:
                raise PreflightError(f"config digest differs: expected {cfg['sha256']}, got {got}")
        observed = _observe_requirements(env_doc)
        done = []
        for check in env_doc["preflight"]:
            PREFLIGHT_CHECKS[check]()
            done.append(check)
        result.update(state="passed", checks=done, observed=observed,
                      environment_sha256=_canon_sha({k: v for k, v in clean.items() if k not in secrets}))
        _write_result(result_path, result)
    except Exception as exc:
        result.update(state="failed", error=f"{type(exc).__name__}: {exc}")
        _write_result(result_path, result)
        raise
    outputs = _outputs(doc)
    rc = run_managed_child(doc["argv"], cwd=doc["cwd"], environment=clean, relay=relay, preemptible=preemptible,
                           import_roots=_import_roots(env_doc), runtime_path=doc["runner_runtime"]["path"],
                           runtime_sha256=doc["runner_runtime"]["sha256"])
    if rc:
        result.update(state="evacuated" if preemptible and rc == EVACUATION_EXIT_CODE else "failed",
                      child_returncode=rc)
        _write_result(result_path, result)
        return rc
    if outputs:
        try:
            _publish_outputs(outputs, clean)
        except Exception as exc:
            result.update(state="failed", error=f"{type(exc).__name__}: {exc}")
            _write_result(result_path, result)
            raise
        result["outputs"] = [o.artifact_id for o in outputs]
    result["state"] = "completed" if outputs else "passed"
    _write_result(result_path, result)
    return 0


def main(argv: Optional[List[str]] = None) -> int:
    args = sys.argv[1:] if argv is None else argv
    if len(args) != 2:
        print("usage: python -m koochak_b200.jobs.runner MANIFEST SHA256", file=sys.stderr)
        return 64
    try:
        return execute_manifest(args[0], args[1])
    except Exception as exc:  # the process error boundary
        print(json.dumps({"kind": "environment_preflight_failed", "error": f"{type(exc).__name__}: {exc}"},
                         sort_keys=True), file=sys.stderr)
        return PREFLIGHT_EXIT_CODE


if __name__ == "__main__":
    raise SystemExit(main())
