"""Node-level GPU health monitor on a CPU thread (reference: koochak/health/background.py:53-204).

At start every rank publishes its device metadata (one ``all_gather_object``);
the lowest rank per hostname becomes that node's leader and polls all of the
node's GPUs with one nvidia-smi query every 30 s. ``failures()`` is cheap
(no GPU, no I/O, no collective): the loop folds it into the per-update
stop-flag reduction. A dead monitor or a sample older than 90 s is itself a
failure.
"""

from __future__ import annotations

import threading
import time
import uuid
from typing import Any

import torch

from .gpu import GpuHealthWatchdog, current_local_rank
from .node_query import QUERY_TIMEOUT_SECONDS, NodeQuery, query_node_samples

__all__ = ["BackgroundGpuHealth", "physical_gpu_uuid", "device_uuid", "INTERVAL_SECONDS", "MAX_SAMPLE_AGE_SECONDS"]

INTERVAL_SECONDS = 30.0
MAX_SAMPLE_AGE_SECONDS = 90.0
JOIN_TIMEOUT_SECONDS = 2 * QUERY_TIMEOUT_SECONDS + 5.0


def physical_gpu_uuid(value: Any) -> str:
    text = value.decode("ascii") if isinstance(value, bytes) else str(value)
    return "GPU-" + str(uuid.UUID(text.removeprefix("GPU-")))


def device_uuid(device: torch.device) -> Any:
    props = torch.cuda.get_device_properties(device)
    value = getattr(props, "uuid", None)
    if value is None:
        raise RuntimeError("this torch build does not expose device UUIDs")
    return value


class BackgroundGpuHealth(GpuHealthWatchdog):
    def __init__(self, **kwargs: Any) -> None:
        super().__init__(**kwargs)
        self.local_rank = current_local_rank()
        self._thread: threading.Thread | None = None
        self._stop = threading.Event()
        self._lock = threading.Lock()
        self._failures: list[dict[str, Any]] = []
        self._watchdogs: list[GpuHealthWatchdog] = []
        self._last_sample_at = time.monotonic()
        self._step = -1
        self._started = False
        self._leader = False
        self._closed = False
        self._sequence = 0
        self._strict_logging = True
        self._query = NodeQuery()
        self.interval_seconds = INTERVAL_SECONDS
        self.max_sample_age_seconds = MAX_SAMPLE_AGE_SECONDS

    def _metadata(self) -> dict[str, Any]:
        err = None
        if self.enabled:
            try:
                self.gpu_query_id = physical_gpu_uuid(device_uuid(self.device))
            except Exception as exc:
                err = f"{type(exc).__name__}: {exc}"
        return {"enabled": self.enabled, "rank": self.rank, "hostname": self.hostname,
                "slurm_node": self.slurm_node, "cuda_device": self.cuda_device, "query_id": self.gpu_query_id,
                "local_rank": self.local_rank, "mapping_error": err}

    def start(self) -> None:
        if self._started:
            return
        self._started = True
        mine = self._metadata()
        peers = [mine]
        if self.world_size > 1 and torch.distributed.is_available() and torch.distributed.is_initialized():
            peers = [None] * self.world_size
            torch.distributed.all_gather_object(peers, mine)
        owned = [p for p in peers if p["enabled"] and p["hostname"] == self.hostname]
        if not owned or self.rank != min(p["rank"] for p in owned):
            return
        self._leader = True
        try:
            self._start_node(owned)
        except Exception as exc:
            self._thread = None
            self._record_error("monitor_start_failed", str(exc))

    def _start_node(self, owned: list[dict[str, Any]]) -> None:
        errors = [p["mapping_error"] for p in owned if p["mapping_error"]]
        if errors:
            self._record_error("monitor_mapping_failed", "; ".join(errors))
            return
        ids = [p["query_id"] for p in owned]
        if len(set(ids)) != len(ids):
            self._record_error("monitor_mapping_failed", "Several ranks name the same GPU")
            return
        for p in owned:
            w = GpuHealthWatchdog(device=torch.device("cuda", p["cuda_device"]), out_dir=self.out_dir, rank=p["rank"],
                                  world_size=self.world_size)
            w.gpu_query_id = p["query_id"]
            w.local_rank = p["local_rank"]
            w._strict_logging = True  # type: ignore[attr-defined]
            self._watchdogs.append(w)
        self._thread = threading.Thread(target=self._poll, name="koochak-gpu-health", daemon=True)
        self._last_sample_at = time.monotonic()
        self._thread.start()

    def update_step(self, step: int) -> None:
        self._step = int(step)

    def failures(self) -> list[dict[str, Any]]:
        if not self._leader:
            return []
        with self._lock:
            failed = bool(self._failures)
            last = self._last_sample_at
        if not failed and not self._closed:
            if self._thread is None or not self._thread.is_alive():
                self._record_error("monitor_died", "GPU health monitor stopped")
            elif time.monotonic() - last > self.max_sample_age_seconds:
                self._record_error("monitor_stale", "GPU health monitor sample is stale")
        with self._lock:
            return list(self._failures)

    def close(self) -> None:
        if self._closed:
            return
        self._stop.set()
        try:
            self._query.cancel()
        except Exception as exc:
            self._record_error("monitor_teardown_failed", f"{type(exc).__name__}: {exc}")
        if self._thread is not None:
            self._thread.join(timeout=JOIN_TIMEOUT_SECONDS)
            if self._thread.is_alive():
                self._record_error("monitor_teardown_failed", "GPU health monitor did not stop")
        self._closed = True

    def _poll(self) -> None:
        try:
            while not self._stop.is_set():
                samples = query_node_samples(self._watchdogs, self._step, run=self._query.run)
                self._sequence += 1
                found = []
                for w, s in zip(self._watchdogs, samples):
                    s.poll_sequence = self._sequence
                    s.poll_monotonic_seconds = time.monotonic()
                    f = w.observe_sample(s)
                    if f is not None:
                        found.append(f.to_dict())
                with self._lock:
                    self._last_sample_at = time.monotonic()
                    self._failures.extend(found)
                    failed = bool(self._failures)
                if failed:
                    return
                self._stop.wait(self.interval_seconds)
        except Exception as exc:
            if not self._stop.is_set():
                self._record_error("monitor_query_failed", f"{type(exc).__name__}: {exc}")

    def _record_error(self, reason: str, message: str) -> None:
        payload = {"event": "gpu_health_monitor_failure", "rank": self.rank, "local_rank": self.local_rank,
                   "hostname": self.hostname, "slurm_node": self.slurm_node, "step": self._step,
                   "timestamp_unix": time.time(), "reasons": [reason], "message": message,
                   "slurm_action": self.slurm_action}
        with self._lock:
            if any(reason in f["reasons"] for f in self._failures):
                return
            self._failures.append(payload)
        try:
            self._append_jsonl("gpu_health_failures", payload)
        except OSError as exc:
            print(f"[gpu-health] could not write monitor failure: {exc}", flush=True)
