"""One nvidia-smi call reads every GPU that a node's monitor is responsible for.

(behaviour of reference koochak/health/node_query.py:22-107)

``NodeQuery`` runs that call as the monitor's only child process, with a
10 s limit, and can kill and reap it from another thread when the monitor
shuts down. ``query_node_samples`` matches the returned rows to the
monitored GPUs (by nvidia-smi index or UUID prefix) and refuses anything it
cannot trust: a missing or ambiguous row, a row without temperature / clock
/ utilization / UUID, negative or non-finite readings, two ranks mapped to
one physical GPU.
"""

from __future__ import annotations

import csv
import math
import subprocess
import threading
from typing import Callable, Dict, List, Optional, Sequence

from .gpu import FALLBACK_QUERY_FIELDS, PRIMARY_QUERY_FIELDS, GpuHealthSample, GpuHealthWatchdog, \
    sample_from_nvidia_smi_row

__all__ = ["NodeQuery", "QUERY_TIMEOUT_SECONDS", "query_node_samples"]

QUERY_TIMEOUT_SECONDS = 10.0


class NodeQuery:
    """Runs one query at a time; ``cancel`` stops the current one and refuses new ones."""

    def __init__(self) -> None:
        self._guard = threading.Lock()
        self._child: Optional[subprocess.Popen] = None
        self._stopped = False

    def _spawn(self, argv: List[str]) -> subprocess.Popen:
        with self._guard:
            if self._stopped:
                raise RuntimeError("GPU health query stopped")
            self._child = subprocess.Popen(argv, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
            return self._child

    def run(self, argv: List[str]) -> subprocess.CompletedProcess:
        child = self._spawn(argv)
        try:
            out, err = child.communicate(timeout=QUERY_TIMEOUT_SECONDS)
        except BaseException:
            child.kill()
            child.communicate()
            raise
        finally:
            with self._guard:
                self._child = None
        return subprocess.CompletedProcess(argv, child.returncode, out, err)

    def cancel(self) -> None:
        with self._guard:
            self._stopped = True
            child = self._child
            if child is not None:
                child.kill()
        if child is not None:
            child.wait(timeout=QUERY_TIMEOUT_SECONDS)


def _row_for(query_id: str, rows: Sequence[Sequence[str]]) -> Sequence[str]:
    def names(row: Sequence[str]) -> bool:
        index, uuid = row[0].strip(), row[1].strip()
        return index == query_id or (query_id.startswith("GPU-") and uuid.startswith(query_id))

    hits = [r for r in rows if names(r)]
    if len(hits) != 1:
        raise RuntimeError(f"GPU health query cannot identify assigned GPU {query_id}")
    return hits[0]


def _finite_non_negative(value: Optional[float]) -> bool:
    return value is not None and math.isfinite(value) and value >= 0


def _checked(w: GpuHealthWatchdog, row: Sequence[str], fields: Sequence[str], step: int) -> GpuHealthSample:
    s = sample_from_nvidia_smi_row(step=step, rank=w.rank, world_size=w.world_size, hostname=w.hostname,
                                   slurm_node=w.slurm_node, cuda_device=w.cuda_device, gpu_query_id=w.gpu_query_id,
                                   fields=fields, row=row)
    s.local_rank = w.local_rank
    if not s.gpu_uuid or not all(_finite_non_negative(v) for v in (s.gpu_temp_c, s.sm_clock_mhz, s.gpu_util_pct)):
        raise RuntimeError(f"GPU health query lacks required values for GPU {w.gpu_query_id}")
    optional = (s.memory_temp_c, s.power_draw_w, s.power_limit_w, s.mem_clock_mhz, s.max_sm_clock_mhz,
                s.mem_util_pct)
    if not all(v is None or _finite_non_negative(v) for v in optional):
        raise RuntimeError(f"GPU health query has invalid readings for GPU {w.gpu_query_id}")
    return s


def query_node_samples(watchdogs: Sequence[GpuHealthWatchdog], step: int, *,
                       run: Callable[[List[str]], subprocess.CompletedProcess]) -> List[GpuHealthSample]:
    """One trusted sample per monitored GPU, in ``watchdogs`` order; ``RuntimeError`` otherwise."""

    exe = watchdogs[0].nvidia_smi
    if exe is None:
        raise RuntimeError("nvidia-smi is not available on PATH")
    selection = ",".join(w.gpu_query_id for w in watchdogs)
    last_error = "nvidia-smi did not return GPU health rows"
    for fields in (PRIMARY_QUERY_FIELDS, FALLBACK_QUERY_FIELDS):
        done = run([exe, "-i", selection, f"--query-gpu={','.join(fields)}", "--format=csv,noheader,nounits"])
        if done.returncode != 0:
            last_error = f"nvidia-smi exited {done.returncode}: {done.stderr.strip()}"
            continue
        rows = list(csv.reader(done.stdout.strip().splitlines()))
        if len(rows) != len(watchdogs) or any(len(r) != len(fields) for r in rows):
            raise RuntimeError("nvidia-smi returned an incomplete GPU health query")
        samples = [_checked(w, _row_for(w.gpu_query_id, rows), fields, step) for w in watchdogs]
        by_uuid: Dict[str, int] = {}
        for s in samples:
            by_uuid[str(s.gpu_uuid)] = by_uuid.get(str(s.gpu_uuid), 0) + 1
        if any(n > 1 for n in by_uuid.values()):
            raise RuntimeError("GPU health query mapped several ranks to the same GPU")
        return samples
    raise RuntimeError(last_error)
