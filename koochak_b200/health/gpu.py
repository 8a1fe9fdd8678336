"""GPU health rules, nvidia-smi sampling, and Slurm recovery (reference: koochak/health/gpu.py:19-630).

A GPU that is busy (utilization >= 80%) fails a sample when it shows a
hardware slowdown, power-brake slowdown, low SM clock (< 70% of max) or
thermal trouble. Non-thermal problems must repeat on 2 consecutive samples;
thermal problems get a 2-hour grace period (continuous, samples at most 5
minutes apart). A confirmed failure makes every rank checkpoint and exit 42,
optionally after asking Slurm to requeue or cancel the job with the bad
nodes excluded (never from inside Scruffy or a nested step).

This module only reads GPU state (nvidia-smi queries); it changes no GPU
setting.
"""

from __future__ import annotations

import csv
import json
import os
import shutil
import socket
import subprocess
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional, Sequence

import torch

from ..utils.paths import canonical_dir

__all__ = ["GpuHealthSample", "GpuHealthFailure", "GpuHealthWatchdog", "evaluate_sample",
           "summarize_failures_for_stdout", "parse_nvidia_smi_csv", "sample_from_nvidia_smi_row",
           "current_local_rank", "current_slurm_node", "query_id_for_cuda_device", "EXIT_CODE",
           "PRIMARY_QUERY_FIELDS", "FALLBACK_QUERY_FIELDS"]

WARMUP_STEPS = 20
CHECK_EVERY_STEPS = 10
REQUIRE_UTILIZATION_PCT = 80.0
CONSECUTIVE_FAILURES = 2
THERMAL_GRACE_SECONDS = 2 * 60 * 60
THERMAL_MAX_SAMPLE_GAP_SECONDS = 5 * 60
THERMAL_REASONS = frozenset({"sw_thermal_slowdown", "hw_thermal_slowdown", "gpu_temp_high", "memory_temp_high"})
MAX_GPU_TEMP_C = 86.0
MAX_MEMORY_TEMP_C = 94.0
MIN_SM_CLOCK_FRAC = 0.70
EXIT_CODE = 42

_REASON_FIELDS = ["clocks_throttle_reasons.active", "clocks_throttle_reasons.sw_thermal_slowdown",
                  "clocks_throttle_reasons.hw_slowdown", "clocks_throttle_reasons.hw_thermal_slowdown",
                  "clocks_throttle_reasons.hw_power_brake_slowdown", "clocks_throttle_reasons.sw_power_cap"]
PRIMARY_QUERY_FIELDS = ["index", "uuid", "name", "temperature.gpu", "temperature.memory", "pstate", "power.draw",
                        "power.limit", "clocks.sm", "clocks.mem", "clocks.max.sm", "utilization.gpu",
                        "utilization.memory", *_REASON_FIELDS]
# Older drivers reject temperature.memory / clocks.max.sm.
FALLBACK_QUERY_FIELDS = ["index", "uuid", "name", "temperature.gpu", "pstate", "power.draw", "power.limit",
                         "clocks.sm", "clocks.mem", "utilization.gpu", "utilization.memory", *_REASON_FIELDS]


def _env_on(name: str) -> bool:
    v = os.environ.get(name)
    return v is not None and v.strip().lower() not in {"", "0", "false", "no", "off"}


def _num(value: Any) -> Optional[float]:
    if value is None:
        return None
    text = str(value).strip()
    if not text or text.upper() == "N/A":
        return None
    try:
        return float(text.split()[0])
    except ValueError:
        return None


def _active(value: Any) -> bool:
    return str(value).strip().lower() == "active"


def _short_host(value: Optional[str]) -> Optional[str]:
    if value is None:
        return None
    text = value.strip()
    return text.split(".")[0] if text else None


def current_slurm_node() -> str:
    return (_short_host(os.environ.get("SLURMD_NODENAME")) or _short_host(os.environ.get("HOSTNAME"))
            or _short_host(socket.gethostname()) or "unknown")


def current_local_rank() -> Optional[int]:
    for key in ("LOCAL_RANK", "SLURM_LOCALID", "MPI_LOCALRANKID", "OMPI_COMM_WORLD_LOCAL_RANK",
                "MV2_COMM_WORLD_LOCAL_RANK"):
        v = os.environ.get(key)
        if v is None:
            continue
        try:
            return int(v)
        except ValueError:
            return None
    return None


def query_id_for_cuda_device(cuda_device: Optional[int]) -> str:
    """nvidia-smi ``-i`` id for a CUDA ordinal, honouring ``CUDA_VISIBLE_DEVICES``."""

    if cuda_device is None:
        return "0"
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        parts = [p.strip() for p in visible.split(",") if p.strip()]
        if 0 <= int(cuda_device) < len(parts):
            return parts[int(cuda_device)]
    return str(int(cuda_device))


@dataclass
class GpuHealthSample:
    step: int
    rank: int
    local_rank: Optional[int]
    world_size: int
    hostname: str
    slurm_node: str
    cuda_device: Optional[int]
    gpu_query_id: str
    gpu_index: Optional[str]
    gpu_uuid: Optional[str]
    gpu_name: Optional[str]
    gpu_temp_c: Optional[float]
    memory_temp_c: Optional[float]
    pstate: Optional[str]
    power_draw_w: Optional[float]
    power_limit_w: Optional[float]
    sm_clock_mhz: Optional[float]
    mem_clock_mhz: Optional[float]
    max_sm_clock_mhz: Optional[float]
    gpu_util_pct: Optional[float]
    mem_util_pct: Optional[float]
    throttle_active_mask: Optional[str]
    sw_thermal_slowdown: bool
    hw_slowdown: bool
    hw_thermal_slowdown: bool
    hw_power_brake_slowdown: bool
    sw_power_cap: bool
    timestamp_unix: float
    poll_sequence: Optional[int] = None
    poll_monotonic_seconds: Optional[float] = None

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)


@dataclass
class GpuHealthFailure:
    sample: GpuHealthSample
    reasons: List[str]
    consecutive_failures: int
    slurm_action: str
    thermal_duration_seconds: float = 0.0

    def to_dict(self) -> Dict[str, Any]:
        out = self.sample.to_dict()
        out.update(event="gpu_health_failure", reasons=list(self.reasons),
                   consecutive_failures=int(self.consecutive_failures), slurm_action=self.slurm_action,
                   thermal_duration_seconds=self.thermal_duration_seconds)
        return out


def sample_from_nvidia_smi_row(*, step: int, rank: int, world_size: int, hostname: str, slurm_node: str,
                               cuda_device: Optional[int], gpu_query_id: str, fields: Sequence[str],
                               row: Sequence[str]) -> GpuHealthSample:
    v = {f: (row[i].strip() if i < len(row) else "N/A") for i, f in enumerate(fields)}
    return GpuHealthSample(
        step=int(step), rank=int(rank), local_rank=current_local_rank(), world_size=int(world_size),
        hostname=hostname, slurm_node=slurm_node, cuda_device=cuda_device, gpu_query_id=gpu_query_id,
        gpu_index=v.get("index"), gpu_uuid=v.get("uuid"), gpu_name=v.get("name"),
        gpu_temp_c=_num(v.get("temperature.gpu")), memory_temp_c=_num(v.get("temperature.memory")),
        pstate=v.get("pstate"), power_draw_w=_num(v.get("power.draw")), power_limit_w=_num(v.get("power.limit")),
        sm_clock_mhz=_num(v.get("clocks.sm")), mem_clock_mhz=_num(v.get("clocks.mem")),
        max_sm_clock_mhz=_num(v.get("clocks.max.sm")), gpu_util_pct=_num(v.get("utilization.gpu")),
        mem_util_pct=_num(v.get("utilization.memory")), throttle_active_mask=v.get("clocks_throttle_reasons.active"),
        sw_thermal_slowdown=_active(v.get("clocks_throttle_reasons.sw_thermal_slowdown")),
        hw_slowdown=_active(v.get("clocks_throttle_reasons.hw_slowdown")),
        hw_thermal_slowdown=_active(v.get("clocks_throttle_reasons.hw_thermal_slowdown")),
        hw_power_brake_slowdown=_active(v.get("clocks_throttle_reasons.hw_power_brake_slowdown")),
        sw_power_cap=_active(v.get("clocks_throttle_reasons.sw_power_cap")), timestamp_unix=time.time())


def parse_nvidia_smi_csv(*, stdout: str, fields: Sequence[str], step: int, rank: int, world_size: int,
                         hostname: str, slurm_node: str, cuda_device: Optional[int],
                         gpu_query_id: str) -> Optional[GpuHealthSample]:
    rows = list(csv.reader(stdout.strip().splitlines())) if stdout.strip() else []
    if not rows:
        return None
    return sample_from_nvidia_smi_row(step=step, rank=rank, world_size=world_size, hostname=hostname,
                                      slurm_node=slurm_node, cuda_device=cuda_device, gpu_query_id=gpu_query_id,
                                      fields=fields, row=rows[0])


def evaluate_sample(sample: GpuHealthSample) -> List[str]:
    """Failure reasons of one sample; an idle GPU (< 80% utilization) never fails."""

    if sample.gpu_util_pct is None or sample.gpu_util_pct < REQUIRE_UTILIZATION_PCT:
        return []
    checks = [
        ("sw_thermal_slowdown", sample.sw_thermal_slowdown),
        ("hw_slowdown", sample.hw_slowdown),
        ("hw_thermal_slowdown", sample.hw_thermal_slowdown),
        ("hw_power_brake_slowdown", sample.hw_power_brake_slowdown),
        ("gpu_temp_high", sample.gpu_temp_c is not None and sample.gpu_temp_c >= MAX_GPU_TEMP_C),
        ("memory_temp_high", sample.memory_temp_c is not None and sample.memory_temp_c >= MAX_MEMORY_TEMP_C),
        ("sm_clock_low", sample.sm_clock_mhz is not None and sample.max_sm_clock_mhz is not None
         and sample.max_sm_clock_mhz > 0 and sample.sm_clock_mhz / sample.max_sm_clock_mhz < MIN_SM_CLOCK_FRAC),
    ]
    return [name for name, hit in checks if hit]


class GpuHealthWatchdog:
    """Per-rank rules state; also the base of the node-level background monitor."""

    def __init__(self, *, device: torch.device, out_dir: str, rank: int, world_size: int) -> None:
        self.device = device
        self.out_dir = canonical_dir(out_dir)
        self.rank = int(rank)
        self.world_size = int(world_size)
        self.hostname = socket.gethostname()
        self.slurm_node = current_slurm_node()
        self.cuda_device = int(device.index) if device.type == "cuda" and device.index is not None else None
        self.local_rank = current_local_rank()
        self.gpu_query_id = query_id_for_cuda_device(self.cuda_device)
        self.nvidia_smi = shutil.which("nvidia-smi")
        self.enabled = device.type == "cuda" and not _env_on("KOOCHAK_GPU_HEALTH_DISABLE")
        self.slurm_disabled = _env_on("KOOCHAK_GPU_HEALTH_SLURM_DISABLE")
        action = os.environ.get("KOOCHAK_GPU_HEALTH_SLURM_ACTION", "exit").strip().lower()
        self.requested_slurm_action = action if action in {"requeue", "cancel", "exit"} else "exit"
        self.slurm_mutation_blocked_reason = self._slurm_mutation_blocked_reason()
        self.slurm_action = "exit" if self.slurm_mutation_blocked_reason else self.requested_slurm_action
        self.exit_code = EXIT_CODE
        self._consecutive_failures = 0
        self._thermal_started_at: Optional[float] = None
        self._thermal_last_sample_at: Optional[float] = None
        self._thermal_samples = 0
        self._notice_written = False

    def should_check_step(self, step: int) -> bool:
        return self.enabled and step >= WARMUP_STEPS and step % CHECK_EVERY_STEPS == 0

    def check_local(self, step: int) -> Optional[GpuHealthFailure]:
        sample = self._query_sample(step)
        if sample is None:
            self._consecutive_failures = 0
            self._thermal_duration(False, time.monotonic())
            return None
        return self.observe_sample(sample)

    def observe_sample(self, sample: GpuHealthSample) -> Optional[GpuHealthFailure]:
        reasons = evaluate_sample(sample)
        thermal = bool(THERMAL_REASONS.intersection(reasons))
        duration = self._thermal_duration(thermal, time.monotonic())
        self._append_jsonl("gpu_health", {**sample.to_dict(), "thermal_duration_seconds": duration,
                                          "thermal_grace_seconds": THERMAL_GRACE_SECONDS})
        # Under thermal throttling, slow clocks and the aggregate HW slowdown
        # flag are consequences; they wait out the thermal grace period too.
        urgent = [r for r in reasons if r not in THERMAL_REASONS
                  and not (thermal and r in {"hw_slowdown", "sm_clock_low"})]
        self._consecutive_failures = self._consecutive_failures + 1 if urgent else 0
        if self._consecutive_failures >= CONSECUTIVE_FAILURES:
            reasons, count = urgent, self._consecutive_failures
        elif thermal and duration >= THERMAL_GRACE_SECONDS and self._thermal_samples >= 2:
            count = self._thermal_samples
        else:
            return None
        failure = GpuHealthFailure(sample=sample, reasons=reasons, consecutive_failures=count,
                                   slurm_action=self.slurm_action, thermal_duration_seconds=duration)
        self._append_jsonl("gpu_health_failures", failure.to_dict())
        return failure

    def _thermal_duration(self, thermal: bool, now: float) -> float:
        if not thermal:
            self._thermal_started_at = self._thermal_last_sample_at = None
            self._thermal_samples = 0
            return 0.0
        if self._thermal_last_sample_at is None or now - self._thermal_last_sample_at > THERMAL_MAX_SAMPLE_GAP_SECONDS:
            self._thermal_started_at = now
            self._thermal_samples = 0
        self._thermal_last_sample_at = now
        self._thermal_samples += 1
        assert self._thermal_started_at is not None
        return now - self._thermal_started_at

    def gather_failures(self, local_failure: Optional[GpuHealthFailure]) -> List[Dict[str, Any]]:
        payload = local_failure.to_dict() if local_failure is not None else None
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            got: List[Optional[Dict[str, Any]]] = [None] * torch.distributed.get_world_size()
            torch.distributed.all_gather_object(got, payload)
            return [g for g in got if g is not None]
        return [payload] if payload is not None else []

    def bad_nodes_from_failures(self, failures: Sequence[Dict[str, Any]]) -> List[str]:
        nodes = set()
        for f in failures:
            node = f.get("slurm_node")
            if not node or str(node).lower() == "unknown":
                node = f.get("hostname")
            if node:
                nodes.add(str(node))
        return self._normalize_against_slurm_nodelist(sorted(nodes))

    def write_failure_summary(self, *, step: int, failures: Sequence[Dict[str, Any]], checkpoint_path: Optional[str],
                              slurm_results: Optional[Sequence[Dict[str, Any]]] = None) -> str:
        summary = {
            "event": "gpu_health_shutdown", "step": int(step), "timestamp_unix": time.time(),
            "checkpoint_path": checkpoint_path, "failures": list(failures),
            "bad_nodes": self.bad_nodes_from_failures(failures), "slurm_job_id": os.environ.get("SLURM_JOB_ID"),
            "slurm_job_name": os.environ.get("SLURM_JOB_NAME"), "slurm_action": self.slurm_action,
            "requested_slurm_action": self.requested_slurm_action,
            "slurm_mutation_blocked_reason": self.slurm_mutation_blocked_reason,
            "slurm_disabled": self.slurm_disabled, "slurm_results": list(slurm_results or []),
        }
        path = self._health_dir() / f"gpu_health_failure_step{step:09d}.json"
        tmp = path.with_suffix(path.suffix + ".tmp")
        tmp.write_text(json.dumps(summary, indent=2, sort_keys=True) + "\n", encoding="utf-8")
        os.replace(tmp, path)
        return str(path)

    def perform_slurm_recovery(self, failures: Sequence[Dict[str, Any]]) -> List[Dict[str, Any]]:
        if self.slurm_disabled or self.slurm_action == "exit":
            return []
        job_id = os.environ.get("SLURM_JOB_ID")
        if not job_id:
            return [{"cmd": "<slurm>", "returncode": None, "stderr": "SLURM_JOB_ID is not set"}]
        bad = self.bad_nodes_from_failures(failures)
        if not bad:
            return [{"cmd": "<slurm>", "returncode": None, "stderr": "no bad nodes reported"}]
        csv_nodes = ",".join(bad)
        results: List[Dict[str, Any]] = []
        if self.slurm_action == "requeue":
            results.append(self._run_command(["scontrol", "update", f"JobId={job_id}", f"ExcNodeList={csv_nodes}"]))
            results.extend(self._exclude_pending_same_name(csv_nodes))
            results.append(self._run_command(["scontrol", "requeue", job_id]))
        elif self.slurm_action == "cancel":
            results.extend(self._exclude_pending_same_name(csv_nodes))
            results.append(self._run_command(["scancel", job_id]))
        return results

    @staticmethod
    def _slurm_mutation_blocked_reason() -> Optional[str]:
        if os.environ.get("SCRUFFY_JOB_ID") or os.environ.get("SCRUFFY_ROOT"):
            return "parent Slurm mutation is forbidden for Scruffy workloads"
        step_id = os.environ.get("SLURM_STEP_ID") or os.environ.get("SLURM_STEPID")
        if step_id and step_id.strip().lower() not in {"batch", "extern"}:
            return f"parent Slurm mutation is forbidden from nested step {step_id}"
        return None

    def _query_sample(self, step: int) -> Optional[GpuHealthSample]:
        if self.nvidia_smi is None:
            self._write_notice("nvidia-smi is not available on PATH")
            return None
        for fields in (PRIMARY_QUERY_FIELDS, FALLBACK_QUERY_FIELDS):
            cmd = [self.nvidia_smi, "-i", self.gpu_query_id, f"--query-gpu={','.join(fields)}",
                   "--format=csv,noheader,nounits"]
            try:
                proc = subprocess.run(cmd, check=False, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                                      timeout=10.0)
            except (OSError, subprocess.SubprocessError) as exc:
                self._write_notice(f"nvidia-smi query failed: {exc}")
                return None
            if proc.returncode != 0:
                continue
            sample = parse_nvidia_smi_csv(stdout=proc.stdout, fields=fields, step=step, rank=self.rank,
                                          world_size=self.world_size, hostname=self.hostname,
                                          slurm_node=self.slurm_node, cuda_device=self.cuda_device,
                                          gpu_query_id=self.gpu_query_id)
            if sample is not None:
                return sample
        self._write_notice("nvidia-smi did not return a parseable GPU health row")
        return None

    def _exclude_pending_same_name(self, csv_nodes: str) -> List[Dict[str, Any]]:
        user, name = os.environ.get("USER"), os.environ.get("SLURM_JOB_NAME")
        if not user or not name:
            return []
        listing = self._run_command(["squeue", "-h", "-u", user, "-t", "PENDING", "-n", name, "-o", "%i"])
        out = [listing]
        if listing.get("returncode") != 0:
            return out
        for jid in str(listing.get("stdout", "")).split():
            out.append(self._run_command(["scontrol", "update", f"JobId={jid}", f"ExcNodeList={csv_nodes}"]))
        return out

    def _normalize_against_slurm_nodelist(self, nodes: Sequence[str]) -> List[str]:
        nodelist = os.environ.get("SLURM_JOB_NODELIST")
        fallback = sorted({_short_host(n) or n for n in nodes})
        if not nodelist:
            return fallback
        res = self._run_command(["scontrol", "show", "hostnames", nodelist])
        if res.get("returncode") != 0:
            return fallback
        names = [ln.strip() for ln in str(res.get("stdout", "")).splitlines() if ln.strip()]
        by_short = {_short_host(n): n for n in names}
        return sorted({by_short.get(_short_host(n), _short_host(n) or n) for n in nodes})

    def _run_command(self, cmd: Sequence[str]) -> Dict[str, Any]:
        try:
            p = subprocess.run(list(cmd), check=False, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                               timeout=20.0)
            return {"cmd": " ".join(cmd), "returncode": p.returncode, "stdout": p.stdout.strip(),
                    "stderr": p.stderr.strip()}
        except (OSError, subprocess.SubprocessError) as exc:
            return {"cmd": " ".join(cmd), "returncode": None, "stdout": "", "stderr": str(exc)}

    def _health_dir(self) -> Path:
        path = Path(self.out_dir) / "gpu_health"
        path.mkdir(parents=True, exist_ok=True)
        return path

    def _append_jsonl(self, stem: str, payload: Dict[str, Any]) -> None:
        try:
            with (self._health_dir() / f"{stem}_rank{self.rank}.jsonl").open("a", encoding="utf-8") as fh:
                fh.write(json.dumps(payload, sort_keys=True) + "\n")
        except OSError as exc:
            if getattr(self, "_strict_logging", False):
                raise
            if stem != "gpu_health_notices" and not self._notice_written:
                self._notice_written = True
                print(f"[gpu-health] failed to write {stem} log: {exc}", flush=True)

    def _write_notice(self, message: str) -> None:
        if self._notice_written:
            return
        self._notice_written = True
        self._append_jsonl("gpu_health_notices", {
            "event": "gpu_health_notice", "rank": self.rank, "hostname": self.hostname,
            "slurm_node": self.slurm_node, "cuda_device": self.cuda_device, "gpu_query_id": self.gpu_query_id,
            "message": message, "timestamp_unix": time.time()})


def summarize_failures_for_stdout(failures: Iterable[Dict[str, Any]]) -> str:
    parts = []
    for f in failures:
        parts.append(
            f"rank={f.get('rank')} local_rank={f.get('local_rank')} host={f.get('hostname')} "
            f"node={f.get('slurm_node')} gpu={f.get('gpu_index')} uuid={f.get('gpu_uuid')} "
            f"reasons={','.join(str(r) for r in f.get('reasons', []))} temp={f.get('gpu_temp_c')}C "
            f"mem={f.get('memory_temp_c')}C sm={f.get('sm_clock_mhz')}/{f.get('max_sm_clock_mhz')}MHz "
            f"util={f.get('gpu_util_pct')}%")
    return " | ".join(parts)
