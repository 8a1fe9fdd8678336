"""Small lifecycle events for an external job coordinator.

(reference: koochak/logging/events.py:362-693)

``make_event_hooks(publish)`` turns training-loop hooks into bounded events
``publish(kind, data)``:

* ``workload.phase``      training started / completed / evacuated / failed
* ``workload.progress``   step, ``completed``/``total`` steps and up to 32 finite
                          scalar metrics (``loss``, ``lr``, ``val_loss`` first),
                          at most once per ``progress_interval_s``
* ``workload.milestone``  evaluation finished, evacuation checkpoint, OOM action
* ``workload.artifact``   a checkpoint, with its publication record (the
                          ``.ready.json`` manifest: path, size, sha256)

Publisher errors warn once and never stop training, except for checkpoint
artifacts when ``strict_artifact_publish`` is set: a downstream scheduler that
waits on that receipt needs the failure (the hook is marked fail-closed).

``make_scruffy_hooks`` binds this to the Scruffy client named by
``SCRUFFY_ROOT`` / ``SCRUFFY_JOB_ID``. Checkpoint artifact events get a
deterministic event id (``koochak-checkpoint-<sha256(artifact_id NUL sha256)>``)
and wait for the coordinator's acknowledgement (default 300 s, env
``KOOCHAK_SCRUFFY_ARTIFACT_ACK_TIMEOUT_SECONDS``). A rejection raises
``CheckpointArtifactAckRejected``; a conflicting use of the id raises
``CheckpointArtifactAckConflict``; an acknowledgement that stays unknown
after reconciliation raises ``CheckpointArtifactAckTimeout`` whose
``exit_code`` (76) tells a scheduler to retry the run with auto-resume.
"""

from __future__ import annotations

import hashlib
import math
import numbers
import os
import time
import warnings
from pathlib import Path
from typing import Any, Callable, Dict, List, Mapping, Optional

from ..core.hooks import rank0_only
from ..interruption import CHECKPOINT_ACK_TIMEOUT_EXIT_CODE
from ..storage import checkpoint as checkpoint_lib

__all__ = [
    "CHECKPOINT_ACK_TIMEOUT_EXIT_CODE", "CHECKPOINT_ACK_TIMEOUT_REASON", "CheckpointArtifactAckError",
    "CheckpointArtifactAckConflict", "CheckpointArtifactAckRejected", "CheckpointArtifactAckTimeout",
    "make_event_hooks", "make_scruffy_hooks",
]

Publish = Callable[[str, Dict[str, object]], object]

MAX_METRICS = 32
MAX_KEY = 96
MAX_PATH = 1024
MAX_ERROR = 512
ACK_TIMEOUT_ENV = "KOOCHAK_SCRUFFY_ARTIFACT_ACK_TIMEOUT_SECONDS"
CHECKPOINT_ACK_TIMEOUT_REASON = "checkpoint_ack_timeout"
_IDENTITY_KEYS = ("v", "artifact_id", "path", "size_bytes", "sha256", "manifest_path")


class CheckpointArtifactAckError(RuntimeError):
    reason = "checkpoint_ack_error"
    retryable = False

    def __init__(self, message: str, *, checkpoint_path: str, event_id: str, publication: Mapping[str, object]):
        super().__init__(message)
        self.checkpoint_path = checkpoint_path
        self.event_id = event_id
        self.publication = dict(publication)


class CheckpointArtifactAckRejected(CheckpointArtifactAckError):
    reason = "checkpoint_ack_rejected"


class CheckpointArtifactAckConflict(CheckpointArtifactAckError):
    reason = "checkpoint_ack_conflict"


class CheckpointArtifactAckTimeout(CheckpointArtifactAckError):
    """The checkpoint exists and is published; only its acknowledgement is unknown."""

    reason = CHECKPOINT_ACK_TIMEOUT_REASON
    retryable = True
    exit_code = CHECKPOINT_ACK_TIMEOUT_EXIT_CODE


# ----------------------------------------------------------------------------- payload helpers

class _Skip:
    pass


_SKIP = _Skip()


def _scalar(v: Any) -> object:
    if hasattr(v, "numel") and hasattr(v, "item"):
        if v.numel() != 1:
            return _SKIP
        v = v.detach().item()
    if isinstance(v, bool):
        return v
    if isinstance(v, numbers.Integral):
        i = int(v)
        return i if -(2 ** 63) <= i < 2 ** 63 else _SKIP
    if isinstance(v, numbers.Real):
        f = float(v)
        return f if math.isfinite(f) else _SKIP
    return _SKIP


def _short(v: object, limit: int) -> str:
    s = str(v)
    return s if len(s) <= limit else s[:limit - 3] + "..."


def _metrics(values: Mapping[str, Any]) -> Dict[str, object]:
    order = {"loss": 0, "lr": 1, "val_loss": 2}
    keys = sorted((k for k in values if isinstance(k, str) and k != "step" and len(k) <= MAX_KEY),
                  key=lambda k: (order.get(k, 3), k))
    out: Dict[str, object] = {}
    for k in keys:
        s = _scalar(values[k])
        if s is _SKIP:
            continue
        out[k] = s
        if len(out) == MAX_METRICS:
            break
    return out


def _step_of(ctx: Mapping[str, Any], values: Optional[Mapping[str, Any]] = None) -> object:
    v = ctx.get("step")
    if v is None and values is not None:
        v = values.get("step")
    s = _scalar(v)
    return None if s is _SKIP else s


def _horizon(ctx: Mapping[str, Any]) -> Optional[int]:
    cfg = ctx.get("train_cfg")
    v = cfg.get("max_steps") if isinstance(cfg, Mapping) else getattr(cfg, "max_steps", None)
    s = _scalar(v)
    return s if type(s) is int and s >= 0 else None


def _publication_or_none(path: str) -> Optional[Dict[str, Any]]:
    try:
        return checkpoint_lib.publication(path)
    except (FileNotFoundError, OSError, ValueError):
        return None  # a checkpoint not written by this runtime: observed, not gated


# ----------------------------------------------------------------------------- hooks

class _Events:
    def __init__(self, publish: Publish, interval: float, clock: Callable[[], float], strict: bool) -> None:
        self.publish, self.interval, self.clock, self.strict = publish, interval, clock, strict
        self.last_progress: Optional[float] = None
        self.last_step: object = None
        self.warned = False

    def send(self, kind: str, data: Dict[str, object], strict: bool = False) -> None:
        try:
            self.publish(kind, data)
        except Exception as exc:
            if strict:
                raise
            if not self.warned:
                self.warned = True
                try:
                    warnings.warn("Koochak event publisher failed; training will continue: "
                                  + _short(exc, MAX_ERROR), RuntimeWarning, stacklevel=2)
                except Exception:
                    pass  # warnings promoted to errors must not stop training either

    def note_step(self, ctx, values=None) -> object:
        s = _step_of(ctx, values)
        if s is not None:
            self.last_step = s
        return s

    def with_step(self, data: Dict[str, object], step: object) -> Dict[str, object]:
        if step is not None:
            data["step"] = step
        return data

    # -- hook bodies
    def on_train_start(self, ctx) -> None:
        self.last_progress, self.last_step = None, None
        data: Dict[str, object] = {"phase": "training", "status": "started"}
        ws = _scalar(ctx.get("world_size"))
        if ws is not _SKIP:
            data["world_size"] = ws
        if ctx.get("device") is not None:
            data["device"] = _short(ctx["device"], 128)
        self.send("workload.phase", data)

    def on_step_end(self, logs, ctx) -> None:
        step = self.note_step(ctx, logs)
        now = float(self.clock())
        if not math.isfinite(now) or (self.last_progress is not None and now - self.last_progress < self.interval):
            return
        self.last_progress = now  # advance first: an unreachable coordinator is not retried every step
        data = self.with_step({"phase": "training", "metrics": _metrics(logs)}, step)
        total = _horizon(ctx)
        if type(step) is int and total is not None:
            data.update(completed=step + 1, total=total, unit="steps")
        self.send("workload.progress", data)

    def on_eval_end(self, metrics, ctx) -> None:
        step = self.note_step(ctx, metrics)
        self.send("workload.milestone", self.with_step(
            {"name": "evaluation_completed", "phase": "evaluation", "metrics": _metrics(metrics)}, step))

    def on_checkpoint(self, path, _ckpt, ctx) -> None:
        step = self.note_step(ctx)
        data = self.with_step({"artifact_type": "checkpoint", "location": _short(path, MAX_PATH)}, step)
        pub = _publication_or_none(path)
        if pub is not None:
            data["publication"] = pub
        self.send("workload.artifact", data, strict=self.strict and pub is not None)

    def on_train_end(self, ctx) -> None:
        step = self.note_step(ctx)
        status = "evacuated" if bool(ctx.get("evacuation_requested", False)) else "completed"
        self.send("workload.phase", self.with_step({"phase": "training", "status": status},
                                                   step if step is not None else self.last_step))

    def on_evacuation(self, path, _ckpt, ctx) -> None:
        step = self.note_step(ctx)
        data = self.with_step({"name": "evacuation_checkpointed", "phase": "training", "status": "checkpointed",
                               "location": _short(path, MAX_PATH)}, step)
        pub = _publication_or_none(path)
        if pub is not None:
            data["publication"] = pub
        self.send("workload.milestone", data)

    def on_oom(self, record, ctx) -> None:
        step = self.note_step(ctx)
        data: Dict[str, object] = {"name": f"oom_{_short(record.get('action'), 32)}", "phase": "training",
                                   "message": _short(record.get("message", ""), MAX_ERROR),
                                   "oom_phase": _short(record.get("phase"), 32)}
        for key in ("consecutive", "skipped_total"):
            s = _scalar(record.get(key))
            if s is not _SKIP:
                data["oom_" + key] = s
        self.send("workload.milestone", self.with_step(data, step))

    def on_exception(self, exc, ctx) -> None:
        step = self.note_step(ctx)
        data = {"phase": "training", "status": "failed", "error_type": _short(type(exc).__name__, 128),
                "message": _short(exc, MAX_ERROR)}
        self.send("workload.phase", self.with_step(data, step if step is not None else self.last_step))


def make_event_hooks(publish: Publish, progress_interval_s: float = 30, clock: Callable[[], float] = time.monotonic,
                     strict_artifact_publish: bool = False) -> Dict[str, List[Callable]]:
    if not callable(publish):
        raise TypeError("publish must be callable")
    interval = float(progress_interval_s)
    if not math.isfinite(interval) or interval < 0:
        raise ValueError("progress_interval_s must be a finite non-negative number")
    if not callable(clock):
        raise TypeError("clock must be callable")
    ev = _Events(publish, interval, clock, bool(strict_artifact_publish))
    ckpt = rank0_only(ev.on_checkpoint)
    if strict_artifact_publish:
        ckpt._koochak_fail_closed = True  # type: ignore[attr-defined]
    return {
        "on_train_start": [rank0_only(ev.on_train_start)],
        "on_step_end": [rank0_only(ev.on_step_end)],
        "on_eval_end": [rank0_only(ev.on_eval_end)],
        "on_checkpoint": [ckpt],
        "on_resume_checkpoint": [rank0_only(ev.on_checkpoint)],  # re-publish durable evidence on resume
        "on_train_end": [rank0_only(ev.on_train_end)],
        "on_evacuation": [rank0_only(ev.on_evacuation)],
        "on_oom": [rank0_only(ev.on_oom)],
        "on_exception": [rank0_only(ev.on_exception)],
    }


# ----------------------------------------------------------------------------- Scruffy binding

def _scruffy_client():
    try:
        import scruffy  # type: ignore
    except ModuleNotFoundError as exc:
        if exc.name == "scruffy":
            raise RuntimeError("Scruffy hooks require the Scruffy client to be importable before training starts; "
                               "declare the client in the execution profile") from exc
        raise RuntimeError("the installed Scruffy client is missing a dependency") from exc
    except ImportError as exc:
        raise RuntimeError("the installed Scruffy client is incompatible") from exc
    fn = getattr(scruffy, "publish_event", None)
    if not callable(fn):
        raise RuntimeError("the installed Scruffy client has no callable publish_event")
    return scruffy, fn


def _same_publication(candidate: object, expected: Mapping[str, object]) -> Optional[bool]:
    if not isinstance(candidate, Mapping):
        return None
    return all(candidate.get(k) == expected.get(k) for k in _IDENTITY_KEYS)


def _job_evidence(job: object, event_id: str, pub: Mapping[str, object]):
    """(accepted, conflict) from a coordinator job view."""

    if not isinstance(job, Mapping):
        return False, False
    items: List[object] = list(job.get("artifact_evidence") or []) if isinstance(job.get("artifact_evidence"), list) else []
    wl = job.get("workload")
    if isinstance(wl, Mapping) and isinstance(wl.get("latest_artifacts"), list):
        items += wl["latest_artifacts"]
    accepted = conflict = False
    for it in items:
        if not isinstance(it, Mapping) or it.get("producer_event_id", it.get("event_id")) != event_id:
            continue
        m = _same_publication(it.get("publication"), pub)
        accepted |= m is True
        conflict |= m is False
    return accepted, conflict


def _looks_like_conflict(exc: BaseException) -> bool:
    return "conflict" in type(exc).__name__.lower() or "already used" in str(exc).lower()


def _reconcile(scruffy, *, root: Path, job_id: str, event_id: str, path: str, pub: Mapping[str, object],
               timeout: float) -> object:
    """Settle an acknowledgement that did not arrive with the publish call."""

    err = dict(checkpoint_path=path, event_id=event_id, publication=pub)
    waiter = getattr(scruffy, "wait_for_event_ack", None)
    if callable(waiter):
        try:
            receipt = waiter(root, job_id=job_id, event_id=event_id, timeout=timeout)
        except TimeoutError:
            receipt = None
        if isinstance(receipt, Mapping):
            if receipt.get("state") == "accepted" or receipt.get("acknowledged") is True:
                return receipt
            if receipt.get("state") == "rejected" or receipt.get("acknowledged") is False:
                raise CheckpointArtifactAckRejected(
                    "Scruffy did not acknowledge checkpoint artifact publication: durably rejected", **err)
        elif isinstance(receipt, tuple) and len(receipt) == 2 and receipt[0]:
            if receipt[1] is not None:
                return receipt
            raise CheckpointArtifactAckRejected(
                "Scruffy did not acknowledge checkpoint artifact publication: durably rejected", **err)
    try:
        from scruffy.storage import report_acknowledged  # type: ignore
    except (ImportError, AttributeError):
        report_acknowledged = None
    if callable(report_acknowledged):
        try:
            acked, identity = report_acknowledged(root, job_id, event_id)
        except Exception as exc:
            if _looks_like_conflict(exc):
                raise CheckpointArtifactAckConflict(
                    "Scruffy receipt evidence conflicts with checkpoint publication", **err) from exc
            acked, identity = False, None
        if acked and identity is None:
            raise CheckpointArtifactAckRejected(
                "Scruffy did not acknowledge checkpoint artifact publication: durably rejected", **err)
        if acked:
            return (acked, identity)
    status = getattr(scruffy, "status", None)
    if callable(status):
        try:
            job = status(root, job_id)
        except (OSError, KeyError, RuntimeError, ValueError, TypeError):
            job = None
        accepted, conflict = _job_evidence(job, event_id, pub)
        if conflict:
            raise CheckpointArtifactAckConflict(
                "Scruffy durable job evidence conflicts with checkpoint publication", **err)
        if accepted:
            return job
    raise CheckpointArtifactAckTimeout(
        "checkpoint artifact acknowledgement deadline expired; durable evidence remains unresolved", **err)


def checkpoint_event_id(pub: Mapping[str, object]) -> Optional[str]:
    aid, digest = pub.get("artifact_id"), pub.get("sha256")
    if not (isinstance(aid, str) and isinstance(digest, str)):
        return None
    return "koochak-checkpoint-" + hashlib.sha256(f"{aid}\0{digest}".encode()).hexdigest()


def make_scruffy_hooks(progress_interval_s: float = 30, clock: Callable[[], float] = time.monotonic,
                       artifact_ack_timeout_s: float | None = None) -> Dict[str, List[Callable]]:
    if artifact_ack_timeout_s is None:
        artifact_ack_timeout_s = os.environ.get(ACK_TIMEOUT_ENV, "300")
    try:
        timeout = float(artifact_ack_timeout_s)
    except (TypeError, ValueError) as exc:
        raise ValueError("artifact_ack_timeout_s must be a finite non-negative number") from exc
    if not math.isfinite(timeout) or timeout < 0:
        raise ValueError("artifact_ack_timeout_s must be a finite non-negative number")
    root = Path(os.environ["SCRUFFY_ROOT"])
    job_id = os.environ["SCRUFFY_JOB_ID"]
    scruffy, publish_event = _scruffy_client()
    source: Dict[str, str] = {"name": "koochak"}
    node = os.environ.get("SCRUFFY_NODE", "").strip()
    if node:
        source["node"] = _short("".join(c if ord(c) >= 32 else "?" for c in node), 256)

    def publish(kind: str, data: Dict[str, object]) -> object:
        pub = data.get("publication")
        gated = kind == "workload.artifact" and isinstance(pub, Mapping)
        event_id = checkpoint_event_id(pub) if gated else None  # type: ignore[arg-type]
        extra: Dict[str, object] = {}
        if event_id is not None:
            extra["event_id"] = event_id
        if gated:
            extra.update(wait=True, timeout=timeout)
        location = str(data.get("location", ""))
        try:
            result = publish_event(root, job_id=job_id, kind=kind, data=data, source=source, **extra)
        except TimeoutError:
            if not gated or event_id is None:
                raise
            return _reconcile(scruffy, root=root, job_id=job_id, event_id=event_id, path=location, pub=pub,
                              timeout=timeout)
        except Exception as exc:
            if gated and event_id is not None and _looks_like_conflict(exc):
                raise CheckpointArtifactAckConflict("Scruffy rejected a conflicting checkpoint artifact event ID",
                                                    checkpoint_path=location, event_id=event_id,
                                                    publication=pub) from exc
            raise
        if gated and event_id is not None:
            if isinstance(result, Mapping):
                if result.get("state") == "accepted" and result.get("acknowledged") is True:
                    return result
                if result.get("state") == "rejected" or result.get("acknowledged") is False:
                    raise CheckpointArtifactAckRejected(
                        "Scruffy did not acknowledge checkpoint artifact publication: "
                        f"rejected (state={result.get('state')!r})",
                        checkpoint_path=location, event_id=event_id, publication=pub)
            return _reconcile(scruffy, root=root, job_id=job_id, event_id=event_id, path=location, pub=pub,
                              timeout=timeout)
        return result

    return make_event_hooks(publish, progress_interval_s=progress_interval_s, clock=clock,
                            strict_artifact_publish=True)
