"""Submission adapters for prepared runs (optional scheduler clients).

(reference: koochak/jobs/backends.py:90-236)

* ``submit_pazuzu(client, prepared, resources=, log_dir=)``: streams every
  artifact to the remote host over the client's ``run`` (a small standard
  library script on the far side checks the digest and publishes it
  immutably), then submits a Slurm job running ``runner_argv()``;
* ``submit_scruffy(prepared, root=, ...)``: stages the run on a shared
  filesystem and enqueues it; a preemptible run needs ``workflow_id`` and
  ``task_id`` because the scheduler honours recovery only for workflow tasks;
* ``submit_scruffy_workflow(workflow, root=)``: stages every task's run,
  then makes the one atomic submission call.

The clients (``pazuzu``, ``scruffy``) are imported only when called.
"""

from __future__ import annotations

import shlex
from inspect import Parameter, signature
from pathlib import Path
from typing import Any, Dict, List, Optional

from .manifest import Artifact, PreparedRun, stage_run
from .workflow import PreparedWorkflow

__all__ = ["submit_pazuzu", "submit_scruffy", "submit_scruffy_workflow", "REMOTE_STAGE"]

# Executed remotely with `python -I -c`; artifact bytes arrive on stdin.
REMOTE_STAGE = r"""
import hashlib, os, pathlib, stat, sys, tempfile
target, want = pathlib.Path(sys.argv[1]), sys.argv[2]
data = sys.stdin.buffer.read()
if hashlib.sha256(data).hexdigest() != want:
    raise SystemExit("artifact digest differs")
target.parent.mkdir(parents=True, exist_ok=True)
def same_as_existing():
    fd = os.open(target, os.O_RDONLY | getattr(os, "O_CLOEXEC", 0) | getattr(os, "O_NOFOLLOW", 0))
    try:
        a = os.fstat(fd)
        if not stat.S_ISREG(a.st_mode):
            raise SystemExit(f"refusing non-regular immutable artifact: {target}")
        buf = b""
        while True:
            c = os.read(fd, 1 << 20)
            if not c:
                break
            buf += c
        b, now = os.fstat(fd), os.lstat(target)
        if not ((a.st_dev, a.st_ino) == (b.st_dev, b.st_ino) == (now.st_dev, now.st_ino)):
            raise SystemExit(f"immutable artifact changed while reading: {target}")
        if buf != data:
            raise SystemExit(f"refusing to replace different artifact: {target}")
        os.fchmod(fd, 0o444)
    finally:
        os.close(fd)
if os.path.lexists(target):
    same_as_existing()
    raise SystemExit(0)
fd, tmp = tempfile.mkstemp(prefix=f".{target.name}.", dir=target.parent)
try:
    with os.fdopen(fd, "wb") as fh:
        fh.write(data); fh.flush(); os.fsync(fh.fileno())
    os.chmod(tmp, 0o444)
    try:
        os.link(tmp, target)
    except FileExistsError:
        same_as_existing()
finally:
    if os.path.exists(tmp):
        os.unlink(tmp)
"""


async def _stage_remote(client: Any, python: str, art: Artifact) -> None:
    cmd = shlex.join([python, "-I", "-c", REMOTE_STAGE, art.path, art.sha256])
    res = await client.run(cmd, stdin=art.content, timeout=60)
    if res.exit_code:
        raise RuntimeError(f"failed to stage {art.path}: {(res.stderr or res.stdout).strip()}")


async def submit_pazuzu(client: Any, prepared: PreparedRun, *, resources: Any, log_dir: str) -> Any:
    try:
        from pazuzu import SlurmJob  # type: ignore
    except ImportError as exc:
        raise RuntimeError("submit_pazuzu requires the optional pazuzu package") from exc
    for art in prepared.artifacts:
        await _stage_remote(client, prepared.python, art)
    job = SlurmJob(name=prepared.name, argv=prepared.runner_argv(), cwd=prepared.cwd, log_dir=log_dir,
                   resources=resources, environment={})
    return await client.submit_slurm(job)


def _scruffy_fn(name: str, caller: str):
    try:
        import scruffy  # type: ignore
    except ModuleNotFoundError as exc:
        if exc.name == "scruffy":
            raise RuntimeError(f"{caller} requires the optional scruffy client") from exc
        raise RuntimeError("the installed scruffy client has a missing dependency") from exc
    except ImportError as exc:
        raise RuntimeError("the installed scruffy client is incompatible with this Python") from exc
    fn = getattr(scruffy, name, None)
    if not callable(fn):
        raise RuntimeError(f"the installed scruffy client has no {name}")
    return fn


def submit_scruffy(prepared: PreparedRun, *, root: str | Path, resources: Any, request_id: str, project_id: str,
                   workflow_id: Optional[str] = None, task_id: Optional[str] = None,
                   needs: Optional[List[Dict[str, str]]] = None,
                   wait_for: Optional[List[Dict[str, str]]] = None) -> Dict[str, Any]:
    recovery = None
    if prepared.preemption is not None:
        if workflow_id is None or task_id is None:
            raise ValueError("preemptible Scruffy jobs need workflow_id and task_id so Scruffy can queue their next "
                             "attempt")
        recovery = prepared.preemption.recovery()
    submit_job = _scruffy_fn("submit_job", "submit_scruffy")
    params = signature(submit_job).parameters
    var_kw = any(p.kind is Parameter.VAR_KEYWORD for p in params.values())
    if wait_for and "wait_for" not in params and not var_kw:
        raise RuntimeError("the installed scruffy client does not support artifact conditions")
    if recovery is not None and "recovery" not in params and not var_kw:
        raise RuntimeError("the installed scruffy client does not support recovery policies")
    stage_run(prepared)
    extra = {"recovery": recovery} if recovery is not None else {}
    return submit_job(Path(root), argv=prepared.runner_argv(), name=prepared.name, cwd=Path(prepared.cwd),
                      environment={}, request=resources, request_id=request_id, project_id=project_id,
                      workflow_id=workflow_id, task_id=task_id, needs=needs, wait_for=wait_for, **extra)


def submit_scruffy_workflow(workflow: PreparedWorkflow, *, root: str | Path) -> Dict[str, Any]:
    if not isinstance(workflow, PreparedWorkflow):
        raise TypeError("workflow must be a PreparedWorkflow")
    submit_workflow = _scruffy_fn("submit_workflow", "submit_scruffy_workflow")
    for t in workflow.tasks:  # every launch manifest is durable before the one submission call
        stage_run(t.run)
    return submit_workflow(Path(root), request_id=workflow.request_id, workflow_id=workflow.workflow_id,
                           project_id=workflow.project_id, tasks=workflow.scruffy_tasks())
