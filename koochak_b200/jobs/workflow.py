"""Workflow (task graph) specifications for the Scruffy scheduler, protocol v1.

(reference: koochak/jobs/workflow.py:120-230)

``PreparedTask`` = one ``PreparedRun`` plus resources, ``needs`` (other tasks
that must be ``succeeded`` or merely ``terminal``), ``wait_for`` (artifacts
of other tasks) and a recovery policy (derived from the run when it was
prepared preemptible; ``evacuated`` retries require that). A
``PreparedWorkflow`` checks that every dependency names a task of the
workflow and that each declared output's provenance names this project,
workflow, task and a code commit; ``scruffy_tasks()`` emits the specs.
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional, Sequence, Tuple

from ..jobs_types import freeze_json, thaw_json
from ..storage.artifact import validate_artifact_id
from .manifest import PREEMPTIBLE_RETRY_ON, PreparedRun

__all__ = ["PreparedTask", "PreparedWorkflow"]

_ID = re.compile(r"[A-Za-z0-9][A-Za-z0-9_.-]{0,127}\Z")


def _ident(v: object, what: str) -> str:
    if not isinstance(v, str) or not _ID.fullmatch(v):
        raise ValueError(f"{what} must be a non-empty scheduler-safe identifier")
    return v


def _objects(v: object, what: str) -> Tuple[Any, ...]:
    if isinstance(v, (str, bytes)) or not isinstance(v, Sequence):
        raise ValueError(f"{what} must be a sequence")
    out = []
    for i, item in enumerate(v):
        if not isinstance(item, Mapping):
            raise ValueError(f"{what}[{i}] must be an object")
        out.append(freeze_json(dict(item), f"{what}[{i}]"))
    return tuple(out)


def _needs(v) -> Tuple[Any, ...]:
    items = _objects(v, "needs")
    for i, it in enumerate(items):
        if set(it) != {"task_id", "condition"}:
            raise ValueError(f"needs[{i}] must contain exactly task_id and condition")
        _ident(it["task_id"], f"needs[{i}].task_id")
        if it["condition"] not in ("succeeded", "terminal"):
            raise ValueError(f"needs[{i}].condition must be 'succeeded' or 'terminal'")
    if len({it["task_id"] for it in items}) != len(items):
        raise ValueError("needs must not contain duplicate task IDs")
    return items


def _wait_for(v) -> Tuple[Any, ...]:
    items = _objects(v, "wait_for")
    for i, it in enumerate(items):
        if set(it) != {"kind", "task_id", "artifact_id"}:
            raise ValueError(f"wait_for[{i}] must contain exactly kind, task_id and artifact_id")
        if it["kind"] != "artifact":
            raise ValueError("wait_for only supports kind='artifact'")
        _ident(it["task_id"], f"wait_for[{i}].task_id")
        validate_artifact_id(it["artifact_id"], f"wait_for[{i}].artifact_id")
    if len({(it["task_id"], it["artifact_id"]) for it in items}) != len(items):
        raise ValueError("wait_for must not contain duplicate artifact conditions")
    return items


def _recovery(v: Optional[Mapping[str, Any]]):
    if v is None:
        return None
    if not isinstance(v, Mapping) or set(v) != {"max_attempts", "retry_on", "evacuation"}:
        raise ValueError("recovery must contain exactly max_attempts, retry_on and evacuation")
    n = v["max_attempts"]
    if type(n) is not int or not 1 <= n <= 10:
        raise ValueError("recovery.max_attempts must be an integer from 1 through 10")
    retry = v["retry_on"]
    if isinstance(retry, (str, bytes)) or not isinstance(retry, Sequence):
        raise ValueError("recovery.retry_on must be a sequence")
    retry = tuple(retry)
    if any(r not in PREEMPTIBLE_RETRY_ON for r in retry):
        raise ValueError(f"recovery.retry_on must use only {sorted(PREEMPTIBLE_RETRY_ON)!r}")
    if len(set(retry)) != len(retry):
        raise ValueError("recovery.retry_on must not contain duplicates")
    ev = v["evacuation"]
    if not isinstance(ev, Mapping) or set(ev) != {"signal", "grace_seconds"}:
        raise ValueError("recovery.evacuation must contain exactly signal and grace_seconds")
    if ev["signal"] != "USR1":
        raise ValueError("recovery.evacuation.signal must equal 'USR1'")
    if type(ev["grace_seconds"]) is not int or ev["grace_seconds"] < 0:
        raise ValueError("recovery.evacuation.grace_seconds must be a non-negative integer")
    return freeze_json({"max_attempts": n, "retry_on": list(retry),
                        "evacuation": {"signal": "USR1", "grace_seconds": ev["grace_seconds"]}}, "recovery")


@dataclass(frozen=True)
class PreparedTask:
    task_id: str
    run: PreparedRun
    resources: Any
    needs: Tuple[Mapping[str, Any], ...] = ()
    wait_for: Tuple[Mapping[str, Any], ...] = ()
    recovery: Optional[Mapping[str, Any]] = None

    def __post_init__(self) -> None:
        _ident(self.task_id, "task_id")
        if not isinstance(self.run, PreparedRun):
            raise TypeError("run must be a PreparedRun")
        res = self.resources.to_dict() if hasattr(self.resources, "to_dict") else self.resources
        if not isinstance(res, Mapping):
            raise ValueError("resources must be a mapping or expose to_dict()")
        rec = self.recovery
        if self.run.preemption is not None:
            if rec is not None:
                raise ValueError("a preemptible run derives its recovery policy; do not also pass recovery")
            rec = self.run.preemption.recovery()
        rec = _recovery(rec)
        if self.run.preemption is None and rec is not None and "evacuated" in rec["retry_on"]:
            raise ValueError("retry_on 'evacuated' requires a run prepared with preemptible=True; "
                             "the runner never forwards evacuation to other runs")
        object.__setattr__(self, "resources", freeze_json(dict(res), "resources"))
        object.__setattr__(self, "needs", _needs(self.needs))
        object.__setattr__(self, "wait_for", _wait_for(self.wait_for))
        object.__setattr__(self, "recovery", rec)

    def to_scruffy_spec(self, *, request_id: str, workflow_id: str, project_id: str) -> Dict[str, Any]:
        spec: Dict[str, Any] = {
            "task_id": self.task_id, "request_id": f"{request_id}/{self.task_id}", "name": self.run.name,
            "argv": self.run.runner_argv(), "cwd": self.run.cwd, "environment": {},
            "resources": thaw_json(self.resources), "needs": [thaw_json(n) for n in self.needs],
            "wait_for": [thaw_json(w) for w in self.wait_for],
        }
        if self.recovery is not None:
            spec["recovery"] = thaw_json(self.recovery)
        return spec


@dataclass(frozen=True)
class PreparedWorkflow:
    request_id: str
    workflow_id: str
    project_id: str
    tasks: Tuple[PreparedTask, ...]

    def __post_init__(self) -> None:
        if not isinstance(self.request_id, str) or not self.request_id.strip() or any(
                ord(c) < 32 for c in self.request_id):
            raise ValueError("request_id must be a non-empty string without control characters")
        _ident(self.workflow_id, "workflow_id")
        _ident(self.project_id, "project_id")
        tasks = tuple(self.tasks)
        if not tasks:
            raise ValueError("workflow must contain at least one task")
        if any(not isinstance(t, PreparedTask) for t in tasks):
            raise TypeError("workflow tasks must be PreparedTask objects")
        ids = [t.task_id for t in tasks]
        if len(set(ids)) != len(ids):
            raise ValueError("workflow task IDs must be unique")
        known = set(ids)
        for t in tasks:
            for n in t.needs:
                if n["task_id"] not in known:
                    raise ValueError(f"missing task dependency: {n['task_id']}")
            for w in t.wait_for:
                if w["task_id"] not in known:
                    raise ValueError(f"missing artifact dependency: {w['task_id']}")
            for out in t.run.declared_outputs:
                want = {"project_id": self.project_id, "workflow_id": self.workflow_id, "task_id": t.task_id}
                for k, v in want.items():
                    if out.provenance.get(k) != v:
                        raise ValueError(f"declared output {out.artifact_id!r} provenance.{k} must equal {v!r}")
                commit = out.provenance.get("code_commit")
                if not isinstance(commit, str) or not commit.strip():
                    raise ValueError(f"declared output {out.artifact_id!r} provenance.code_commit must be non-empty")
        object.__setattr__(self, "tasks", tasks)

    def scruffy_tasks(self) -> List[Dict[str, Any]]:
        return [t.to_scruffy_spec(request_id=self.request_id, workflow_id=self.workflow_id,
                                  project_id=self.project_id) for t in self.tasks]
