"""One nvidia-smi query for all GPUs a node monitor owns (reference: koochak/health/node_query.py:22-107)."""

from __future__ import annotations

import csv
import math
import subprocess
import threading
from typing import Callable, Sequence

from .gpu import FALLBACK_QUERY_FIELDS, PRIMARY_QUERY_FIELDS, GpuHealthSample, GpuHealthWatchdog, \
    sample_from_nvidia_smi_row

__all__ = ["NodeQuery", "QUERY_TIMEOUT_SECONDS", "query_node_samples"]

QUERY_TIMEOUT_SECONDS = 10.0


class NodeQuery:
    """Owns the monitor's single child process; ``cancel`` kills and reaps it."""

    def __init__(self) -> None:
        self._lock = threading.Lock()
        self._proc: subprocess.Popen | None = None
        self._closing = False

    def run(self, argv: list[str]) -> subprocess.CompletedProcess:
        with self._lock:
            if self._closing:
                raise RuntimeError("GPU health query stopped")
            proc = subprocess.Popen(argv, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
            self._proc = proc
        try:
            out, err = proc.communicate(timeout=QUERY_TIMEOUT_SECONDS)
            return subprocess.CompletedProcess(argv, proc.returncode, out, err)
        except BaseException:
            proc.kill()
            proc.communicate()
            raise
        finally:
            with self._lock:
                self._proc = None

    def cancel(self) -> None:
        with self._lock:
            self._closing = True
            proc = self._proc
            if proc is not None:
                proc.kill()
        if proc is not None:
            proc.wait(timeout=QUERY_TIMEOUT_SECONDS)


def query_node_samples(watchdogs: Sequence[GpuHealthWatchdog], step: int, *,
                       run: Callable[[list[str]], subprocess.CompletedProcess]) -> list[GpuHealthSample]:
    """One parseable, distinct row per assigned physical GPU, or RuntimeError."""

    exe = watchdogs[0].nvidia_smi
    if exe is None:
        raise RuntimeError("nvidia-smi is not available on PATH")
    ids = [w.gpu_query_id for w in watchdogs]
    error = "nvidia-smi did not return GPU health rows"
    for fields in (PRIMARY_QUERY_FIELDS, FALLBACK_QUERY_FIELDS):
        proc = run([exe, "-i", ",".join(ids), f"--query-gpu={','.join(fields)}", "--format=csv,noheader,nounits"])
        if proc.returncode != 0:
            error = f"nvidia-smi exited {proc.returncode}: {proc.stderr.strip()}"
            continue
        rows = list(csv.reader(proc.stdout.strip().splitlines()))
        if len(rows) != len(watchdogs) or any(len(r) != len(fields) for r in rows):
            raise RuntimeError("nvidia-smi returned an incomplete GPU health query")
        samples = [_sample_for(w, rows, fields, step) for w in watchdogs]
        if len({s.gpu_uuid for s in samples}) != len(samples):
            raise RuntimeError("GPU health query mapped several ranks to the same GPU")
        return samples
    raise RuntimeError(error)


def _sample_for(w: GpuHealthWatchdog, rows, fields, step) -> GpuHealthSample:
    qid = w.gpu_query_id
    hits = [r for r in rows if r[0].strip() == qid or (qid.startswith("GPU-") and r[1].strip().startswith(qid))]
    if len(hits) != 1:
        raise RuntimeError(f"GPU health query cannot identify assigned GPU {qid}")
    s = sample_from_nvidia_smi_row(step=step, rank=w.rank, world_size=w.world_size, hostname=w.hostname,
                                   slurm_node=w.slurm_node, cuda_device=w.cuda_device, gpu_query_id=qid,
                                   fields=fields, row=hits[0])
    s.local_rank = w.local_rank
    required = (s.gpu_temp_c, s.sm_clock_mhz, s.gpu_util_pct)
    if any(v is None or not math.isfinite(v) or v < 0 for v in required) or not s.gpu_uuid:
        raise RuntimeError(f"GPU health query lacks required values for GPU {qid}")
    optional = (s.memory_temp_c, s.power_draw_w, s.power_limit_w, s.mem_clock_mhz, s.max_sm_clock_mhz, s.mem_util_pct)
    if any(v is not None and (not math.isfinite(v) or v < 0) for v in optional):
        raise RuntimeError(f"GPU health query has invalid readings for GPU {qid}")
    return s
