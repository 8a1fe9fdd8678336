"""A per-node GPU-health monitor that runs on a CPU thread, out of the training loop's way.

(behaviour of reference koochak/health/background.py:53-204)

Start-up (``start``, on every rank, one ``all_gather_object``): each rank
publishes which physical GPU it drives (its UUID, read here on the main
thread) and its host name. On every host the lowest enabled rank becomes the
leader (``elect_leader``); only the leader starts the thread, which queries
all of that host's GPUs with one nvidia-smi call every ``interval_seconds``
(30 s) and feeds each GPU's rules state (``GpuHealthWatchdog``).

Per update (``failures``): no GPU work, no I/O, no collective -- the loop
folds a non-empty answer into its per-update stop-flag reduction. A monitor
that died, or whose newest sample is older than ``max_sample_age_seconds``
(90 s), counts as a failure itself, as does a query that raised.

``close`` cancels a running query, stops the thread and waits for it.
"""

from __future__ import annotations

import threading
import time
import uuid
from typing import Any, Callable, Dict, List, Optional, Sequence

import torch

from .gpu import GpuHealthWatchdog, current_local_rank
from .node_query import QUERY_TIMEOUT_SECONDS, NodeQuery, query_node_samples

__all__ = ["BackgroundGpuHealth", "physical_gpu_uuid", "device_uuid", "elect_leader", "INTERVAL_SECONDS",
           "MAX_SAMPLE_AGE_SECONDS"]

INTERVAL_SECONDS = 30.0
MAX_SAMPLE_AGE_SECONDS = 90.0
JOIN_TIMEOUT_SECONDS = 2 * QUERY_TIMEOUT_SECONDS + 5.0


def physical_gpu_uuid(value: Any) -> str:
    """``GPU-<canonical uuid>`` from a torch device UUID (bytes or text, with or without the prefix)."""

    text = value.decode("ascii") if isinstance(value, bytes) else str(value)
    if text.startswith("GPU-"):
        text = text[4:]
    return f"GPU-{uuid.UUID(text)}"


def device_uuid(device: torch.device) -> Any:
    found = getattr(torch.cuda.get_device_properties(device), "uuid", None)
    if found is None:
        raise RuntimeError("this torch build does not expose device UUIDs")
    return found


def elect_leader(peers: Sequence[Dict[str, Any]], rank: int, hostname: str) -> Optional[List[Dict[str, Any]]]:
    """The enabled peers on ``hostname`` when ``rank`` is the lowest of them (this rank leads), else None."""

    local = [p for p in peers if p["enabled"] and p["hostname"] == hostname]
    if local and rank == min(p["rank"] for p in local):
        return sorted(local, key=lambda p: p["rank"])
    return None


class _FailureBook:
    """Thread-safe record of monitor failures (one per reason) and of the newest sample time."""

    def __init__(self, clock: Callable[[], float]) -> None:
        self._lock = threading.Lock()
        self._items: List[Dict[str, Any]] = []
        self.clock = clock
        self.last_sample = clock()

    def add(self, items: Sequence[Dict[str, Any]], sampled: bool = False) -> bool:
        """Record ``items`` (and a fresh sample time); True once any failure is on record."""

        with self._lock:
            if sampled:
                self.last_sample = self.clock()
            self._items.extend(items)
            return bool(self._items)

    def add_once(self, item: Dict[str, Any]) -> bool:
        reason = item["reasons"][0]
        with self._lock:
            if any(reason in f["reasons"] for f in self._items):
                return False
            self._items.append(item)
            return True

    def snapshot(self):
        with self._lock:
            return list(self._items), self.last_sample


class BackgroundGpuHealth(GpuHealthWatchdog):
    interval_seconds = INTERVAL_SECONDS
    max_sample_age_seconds = MAX_SAMPLE_AGE_SECONDS

    def __init__(self, **kwargs: Any) -> None:
        super().__init__(**kwargs)
        self.local_rank = current_local_rank()
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._book = _FailureBook(time.monotonic)
        self._node: List[GpuHealthWatchdog] = []
        self._query = NodeQuery()
        self._step = -1
        self._sequence = 0
        self._started = self._leader = self._closed = False

    # Seams a test may replace (class attributes, so they apply to the instance the loop builds).
    query_node = staticmethod(query_node_samples)
    read_uuid = staticmethod(device_uuid)

    def _describe(self) -> Dict[str, Any]:
        error = None
        if self.enabled:
            try:
                self.gpu_query_id = physical_gpu_uuid(self.read_uuid(self.device))
            except Exception as exc:  # reported by the leader as a mapping failure
                error = f"{type(exc).__name__}: {exc}"
        return {"enabled": self.enabled, "rank": self.rank, "hostname": self.hostname, "slurm_node": self.slurm_node,
                "cuda_device": self.cuda_device, "query_id": self.gpu_query_id, "local_rank": self.local_rank,
                "mapping_error": error}

    def start(self) -> None:
        if self._started:
            return
        self._started = True
        me = self._describe()
        peers: List[Any] = [me]
        if self.world_size > 1 and torch.distributed.is_available() and torch.distributed.is_initialized():
            peers = [None] * self.world_size
            torch.distributed.all_gather_object(peers, me)
        node = elect_leader(peers, self.rank, self.hostname)
        if node is None:
            return
        self._leader = True
        try:
            self._launch(node)
        except Exception as exc:
            self._thread = None
            self._fail("monitor_start_failed", str(exc))

    def _launch(self, node: List[Dict[str, Any]]) -> None:
        problems = [p["mapping_error"] for p in node if p["mapping_error"]]
        ids = [p["query_id"] for p in node]
        if problems or len(set(ids)) != len(ids):
            self._fail("monitor_mapping_failed", "; ".join(problems) or "Several ranks name the same GPU")
            return
        for p in node:
            w = GpuHealthWatchdog(device=torch.device("cuda", p["cuda_device"]), out_dir=self.out_dir, rank=p["rank"],
                                  world_size=self.world_size)
            w.gpu_query_id, w.local_rank = p["query_id"], p["local_rank"]
            w.log.strict = True
            self._node.append(w)
        self._book.add([], sampled=True)
        self._thread = threading.Thread(target=self._loop, name="koochak-gpu-health", daemon=True)
        self._thread.start()

    def update_step(self, step: int) -> None:
        self._step = int(step)

    def failures(self) -> List[Dict[str, Any]]:
        if not self._leader:
            return []
        found, last = self._book.snapshot()
        if not found and not self._closed:
            if self._thread is None or not self._thread.is_alive():
                self._fail("monitor_died", "GPU health monitor stopped")
            elif time.monotonic() - last > self.max_sample_age_seconds:
                self._fail("monitor_stale", "GPU health monitor sample is stale")
        return self._book.snapshot()[0]

    def close(self) -> None:
        if self._closed:
            return
        self._stop.set()
        try:
            self._query.cancel()
        except Exception as exc:
            self._fail("monitor_teardown_failed", f"{type(exc).__name__}: {exc}")
        if self._thread is not None:
            self._thread.join(timeout=JOIN_TIMEOUT_SECONDS)
            if self._thread.is_alive():
                self._fail("monitor_teardown_failed", "GPU health monitor did not stop")
        self._closed = True

    def _poll_once(self) -> bool:
        samples = self.query_node(self._node, self._step, run=self._query.run)
        self._sequence += 1
        failed = []
        for w, s in zip(self._node, samples):
            s.poll_sequence, s.poll_monotonic_seconds = self._sequence, time.monotonic()
            verdict = w.observe_sample(s)
            if verdict is not None:
                failed.append(verdict.to_dict())
        return self._book.add(failed, sampled=True)

    def _loop(self) -> None:
        try:
            while not self._stop.is_set():
                if self._poll_once():
                    return  # a failure is on record: the loop stops every rank
                self._stop.wait(self.interval_seconds)
        except Exception as exc:
            if not self._stop.is_set():
                self._fail("monitor_query_failed", f"{type(exc).__name__}: {exc}")

    def _fail(self, reason: str, message: str) -> None:
        record = {"event": "gpu_health_monitor_failure", "rank": self.rank, "local_rank": self.local_rank,
                  "hostname": self.hostname, "slurm_node": self.slurm_node, "step": self._step,
                  "timestamp_unix": time.time(), "reasons": [reason], "message": message,
                  "slurm_action": self.slurm_action}
        if not self._book.add_once(record):
            return
        try:
            self.log.append("gpu_health_failures", record)
        except OSError as exc:
            print(f"[gpu-health] could not write monitor failure: {exc}", flush=True)
