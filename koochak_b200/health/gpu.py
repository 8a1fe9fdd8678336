"""GPU health: nvidia-smi readings, the rules that call a GPU unhealthy, and what a failure triggers.

(behaviour of reference koochak/health/gpu.py:19-630)

Rules (``evaluate_sample``). Only a busy GPU (utilization >= 80%) is judged.
It fails a sample for any of: software or hardware thermal slowdown, the
aggregate hardware slowdown flag, the power-brake slowdown, GPU temperature
>= 86 C, memory temperature >= 94 C, or an SM clock below 70% of its maximum.
``sw_power_cap`` alone is normal on a power-capped part and never fails.

Verdicts (``_Verdicts``). Non-thermal reasons must repeat on two consecutive
samples. Thermal reasons are a slow problem: they fail only after two hours
of continuous thermal evidence (samples at most five minutes apart, measured
on the monotonic clock). While a GPU is thermally limited its slow clock and
the aggregate slowdown flag are consequences, not separate faults; the power
brake stays fast.

Consequences (``SlurmRecovery``). A confirmed failure makes every rank
checkpoint and exit 42. Optionally (``KOOCHAK_GPU_HEALTH_SLURM_ACTION``
``requeue`` / ``cancel``; default ``exit``) rank 0 asks Slurm to requeue or
cancel the job with the bad nodes excluded -- never from inside a Scruffy
workload or a nested job step, and never when
``KOOCHAK_GPU_HEALTH_SLURM_DISABLE`` is set.

This module only reads GPU state; it changes no GPU setting. Time and
command execution are injectable (``clock``, ``runner``) so every rule and
Slurm action is testable without a GPU or a scheduler.
"""

from __future__ import annotations

import csv
import json
import os
import shutil
import socket
import subprocess
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import torch

from ..utils.paths import canonical_dir

__all__ = ["GpuHealthSample", "GpuHealthFailure", "GpuHealthWatchdog", "SlurmRecovery", "Thresholds",
           "evaluate_sample", "summarize_failures_for_stdout", "parse_nvidia_smi_csv", "sample_from_nvidia_smi_row",
           "current_local_rank", "current_slurm_node", "query_id_for_cuda_device", "EXIT_CODE",
           "PRIMARY_QUERY_FIELDS", "FALLBACK_QUERY_FIELDS", "THERMAL_GRACE_SECONDS",
           "THERMAL_MAX_SAMPLE_GAP_SECONDS", "THERMAL_REASONS"]


@dataclass(frozen=True)
class Thresholds:
    busy_util_pct: float = 80.0
    max_gpu_temp_c: float = 86.0
    max_memory_temp_c: float = 94.0
    min_sm_clock_frac: float = 0.70
    consecutive: int = 2
    thermal_grace_s: float = 2 * 60 * 60
    thermal_max_gap_s: float = 5 * 60


DEFAULT = Thresholds()
WARMUP_STEPS = 20
CHECK_EVERY_STEPS = 10
EXIT_CODE = 42
THERMAL_GRACE_SECONDS = int(DEFAULT.thermal_grace_s)
THERMAL_MAX_SAMPLE_GAP_SECONDS = int(DEFAULT.thermal_max_gap_s)
THERMAL_REASONS = frozenset({"sw_thermal_slowdown", "hw_thermal_slowdown", "gpu_temp_high", "memory_temp_high"})
_THERMAL_CONSEQUENCES = frozenset({"hw_slowdown", "sm_clock_low"})

# nvidia-smi --query-gpu fields, in the order the CSV columns come back.
_THROTTLE = ["clocks_throttle_reasons.active", "clocks_throttle_reasons.sw_thermal_slowdown",
             "clocks_throttle_reasons.hw_slowdown", "clocks_throttle_reasons.hw_thermal_slowdown",
             "clocks_throttle_reasons.hw_power_brake_slowdown", "clocks_throttle_reasons.sw_power_cap"]
PRIMARY_QUERY_FIELDS = ["index", "uuid", "name", "temperature.gpu", "temperature.memory", "pstate", "power.draw",
                        "power.limit", "clocks.sm", "clocks.mem", "clocks.max.sm", "utilization.gpu",
                        "utilization.memory", *_THROTTLE]
# For drivers that reject temperature.memory and clocks.max.sm.
FALLBACK_QUERY_FIELDS = [f for f in PRIMARY_QUERY_FIELDS if f not in ("temperature.memory", "clocks.max.sm")]


# ----------------------------------------------------------------------------- environment


def _env_flag(name: str) -> bool:
    raw = os.environ.get(name)
    return raw is not None and raw.strip().lower() not in {"", "0", "false", "no", "off"}


def _short_host(value: Optional[str]) -> Optional[str]:
    text = (value or "").strip()
    return text.split(".", 1)[0] if text else None


def current_slurm_node() -> str:
    for candidate in (os.environ.get("SLURMD_NODENAME"), os.environ.get("HOSTNAME"), socket.gethostname()):
        short = _short_host(candidate)
        if short:
            return short
    return "unknown"


def current_local_rank() -> Optional[int]:
    """The first launcher variable naming a local rank (``None`` if absent or not an integer)."""

    for key in ("LOCAL_RANK", "SLURM_LOCALID", "MPI_LOCALRANKID", "OMPI_COMM_WORLD_LOCAL_RANK",
                "MV2_COMM_WORLD_LOCAL_RANK"):
        if key in os.environ:
            try:
                return int(os.environ[key])
            except ValueError:
                return None
    return None


def query_id_for_cuda_device(cuda_device: Optional[int]) -> str:
    """nvidia-smi ``-i`` id of a CUDA ordinal, through ``CUDA_VISIBLE_DEVICES`` when it is set."""

    if cuda_device is None:
        return "0"
    visible = [p.strip() for p in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if p.strip()]
    index = int(cuda_device)
    return visible[index] if 0 <= index < len(visible) else str(index)


# ----------------------------------------------------------------------------- samples


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
        record = self.sample.to_dict()
        record["event"] = "gpu_health_failure"
        record["reasons"] = list(self.reasons)
        record["consecutive_failures"] = int(self.consecutive_failures)
        record["slurm_action"] = self.slurm_action
        record["thermal_duration_seconds"] = self.thermal_duration_seconds
        return record


def _number(text: Optional[str]) -> Optional[float]:
    """First token of an nvidia-smi value as a float (``N/A``, blanks and junk: ``None``)."""

    words = (text or "").split()
    if not words or words[0].upper() == "N/A":
        return None
    try:
        return float(words[0])
    except ValueError:
        return None


def _flag(text: Optional[str]) -> bool:
    return (text or "").strip().lower() == "active"


def _text(text: Optional[str]) -> Optional[str]:
    return text


# Sample attribute <- (nvidia-smi field, parser).
_COLUMNS: Dict[str, Tuple[str, Callable[[Optional[str]], Any]]] = {
    "gpu_index": ("index", _text), "gpu_uuid": ("uuid", _text), "gpu_name": ("name", _text),
    "gpu_temp_c": ("temperature.gpu", _number), "memory_temp_c": ("temperature.memory", _number),
    "pstate": ("pstate", _text), "power_draw_w": ("power.draw", _number), "power_limit_w": ("power.limit", _number),
    "sm_clock_mhz": ("clocks.sm", _number), "mem_clock_mhz": ("clocks.mem", _number),
    "max_sm_clock_mhz": ("clocks.max.sm", _number), "gpu_util_pct": ("utilization.gpu", _number),
    "mem_util_pct": ("utilization.memory", _number), "throttle_active_mask": ("clocks_throttle_reasons.active", _text),
    "sw_thermal_slowdown": ("clocks_throttle_reasons.sw_thermal_slowdown", _flag),
    "hw_slowdown": ("clocks_throttle_reasons.hw_slowdown", _flag),
    "hw_thermal_slowdown": ("clocks_throttle_reasons.hw_thermal_slowdown", _flag),
    "hw_power_brake_slowdown": ("clocks_throttle_reasons.hw_power_brake_slowdown", _flag),
    "sw_power_cap": ("clocks_throttle_reasons.sw_power_cap", _flag),
}


def sample_from_nvidia_smi_row(*, step: int, rank: int, world_size: int, hostname: str, slurm_node: str,
                               cuda_device: Optional[int], gpu_query_id: str, fields: Sequence[str],
                               row: Sequence[str]) -> GpuHealthSample:
    """A sample from one CSV row whose columns are ``fields`` (missing columns read as ``N/A``)."""

    cells = dict(zip(fields, (c.strip() for c in row)))
    readings = {attr: parse(cells.get(name, "N/A")) for attr, (name, parse) in _COLUMNS.items()}
    return GpuHealthSample(step=int(step), rank=int(rank), local_rank=current_local_rank(),
                           world_size=int(world_size), hostname=hostname, slurm_node=slurm_node,
                           cuda_device=cuda_device, gpu_query_id=gpu_query_id, timestamp_unix=time.time(),
                           **readings)


def parse_nvidia_smi_csv(*, stdout: str, fields: Sequence[str], step: int, rank: int, world_size: int,
                         hostname: str, slurm_node: str, cuda_device: Optional[int],
                         gpu_query_id: str) -> Optional[GpuHealthSample]:
    """The sample of the first CSV row of ``stdout`` (``None`` when there is none)."""

    rows = [r for r in csv.reader(stdout.strip().splitlines())] if stdout.strip() else []
    if not rows:
        return None
    return sample_from_nvidia_smi_row(step=step, rank=rank, world_size=world_size, hostname=hostname,
                                      slurm_node=slurm_node, cuda_device=cuda_device, gpu_query_id=gpu_query_id,
                                      fields=fields, row=rows[0])


# ----------------------------------------------------------------------------- rules


def _clock_low(s: GpuHealthSample, th: Thresholds) -> bool:
    if s.sm_clock_mhz is None or not s.max_sm_clock_mhz:
        return False
    return s.max_sm_clock_mhz > 0 and s.sm_clock_mhz < th.min_sm_clock_frac * s.max_sm_clock_mhz


def _at_least(value: Optional[float], limit: float) -> bool:
    return value is not None and value >= limit


_RULES: List[Tuple[str, Callable[[GpuHealthSample, Thresholds], bool]]] = [
    ("sw_thermal_slowdown", lambda s, th: s.sw_thermal_slowdown),
    ("hw_slowdown", lambda s, th: s.hw_slowdown),
    ("hw_thermal_slowdown", lambda s, th: s.hw_thermal_slowdown),
    ("hw_power_brake_slowdown", lambda s, th: s.hw_power_brake_slowdown),
    ("gpu_temp_high", lambda s, th: _at_least(s.gpu_temp_c, th.max_gpu_temp_c)),
    ("memory_temp_high", lambda s, th: _at_least(s.memory_temp_c, th.max_memory_temp_c)),
    ("sm_clock_low", _clock_low),
]


def evaluate_sample(sample: GpuHealthSample, thresholds: Thresholds = DEFAULT) -> List[str]:
    """Failure reasons of one sample, in a fixed order; an idle GPU never fails."""

    if not _at_least(sample.gpu_util_pct, thresholds.busy_util_pct):
        return []
    return [reason for reason, broken in _RULES if broken(sample, thresholds)]


@dataclass
class _Verdicts:
    """Turns per-sample reasons into failures: two in a row for faults, a long episode for heat."""

    thresholds: Thresholds = DEFAULT
    streak: int = 0
    episode_start: Optional[float] = None
    episode_last: Optional[float] = None
    episode_samples: int = 0

    def clear(self) -> None:
        self.streak = 0
        self.episode_start = self.episode_last = None
        self.episode_samples = 0

    def _heat(self, hot: bool, now: float) -> float:
        if not hot:
            self.episode_start = self.episode_last = None
            self.episode_samples = 0
            return 0.0
        broken_run = self.episode_last is None or now - self.episode_last > self.thresholds.thermal_max_gap_s
        if broken_run:
            self.episode_start, self.episode_samples = now, 0
        self.episode_last = now
        self.episode_samples += 1
        return now - float(self.episode_start)

    def judge(self, reasons: List[str], now: float) -> Tuple[Optional[Tuple[List[str], int]], float]:
        """((failure reasons, count) or None, thermal episode length so far)."""

        hot = any(r in THERMAL_REASONS for r in reasons)
        duration = self._heat(hot, now)
        faults = [r for r in reasons
                  if r not in THERMAL_REASONS and not (hot and r in _THERMAL_CONSEQUENCES)]
        self.streak = self.streak + 1 if faults else 0
        if self.streak >= self.thresholds.consecutive:
            return (faults, self.streak), duration
        if hot and duration >= self.thresholds.thermal_grace_s and self.episode_samples >= 2:
            return (reasons, self.episode_samples), duration
        return None, duration


# ----------------------------------------------------------------------------- Slurm


def _run(cmd: Sequence[str]) -> Dict[str, Any]:
    shown = " ".join(cmd)
    try:
        done = subprocess.run(list(cmd), check=False, capture_output=True, text=True, timeout=20.0)
    except (OSError, subprocess.SubprocessError) as exc:
        return {"cmd": shown, "returncode": None, "stdout": "", "stderr": str(exc)}
    return {"cmd": shown, "returncode": done.returncode, "stdout": done.stdout.strip(), "stderr": done.stderr.strip()}


@dataclass
class SlurmRecovery:
    """What rank 0 asks Slurm to do about bad nodes, from the environment at start-up."""

    requested_action: str = "exit"
    disabled: bool = False
    blocked_reason: Optional[str] = None
    runner: Callable[[Sequence[str]], Dict[str, Any]] = field(default=_run, repr=False)

    @classmethod
    def from_env(cls, runner: Optional[Callable[[Sequence[str]], Dict[str, Any]]] = None) -> "SlurmRecovery":
        wanted = os.environ.get("KOOCHAK_GPU_HEALTH_SLURM_ACTION", "exit").strip().lower()
        return cls(requested_action=wanted if wanted in {"requeue", "cancel", "exit"} else "exit",
                   disabled=_env_flag("KOOCHAK_GPU_HEALTH_SLURM_DISABLE"), blocked_reason=cls._blocked(),
                   runner=runner or _run)

    @staticmethod
    def _blocked() -> Optional[str]:
        if os.environ.get("SCRUFFY_JOB_ID") or os.environ.get("SCRUFFY_ROOT"):
            return "parent Slurm mutation is forbidden for Scruffy workloads"
        step = os.environ.get("SLURM_STEP_ID") or os.environ.get("SLURM_STEPID")
        if step and step.strip().lower() not in {"batch", "extern"}:
            return f"parent Slurm mutation is forbidden from nested step {step}"
        return None

    @property
    def action(self) -> str:
        return "exit" if self.blocked_reason else self.requested_action

    def node_names(self, nodes: Sequence[str]) -> List[str]:
        """Node names as Slurm spells them in this job's node list (short host names otherwise)."""

        short = sorted({_short_host(n) or n for n in nodes})
        nodelist = os.environ.get("SLURM_JOB_NODELIST")
        if not nodelist:
            return short
        listing = self.runner(["scontrol", "show", "hostnames", nodelist])
        if listing.get("returncode") != 0:
            return short
        known = {_short_host(h): h for h in (ln.strip() for ln in str(listing.get("stdout", "")).splitlines()) if h}
        return sorted({known.get(_short_host(n), _short_host(n) or n) for n in nodes})

    def _exclude_from_pending_twins(self, nodes_csv: str) -> List[Dict[str, Any]]:
        user, name = os.environ.get("USER"), os.environ.get("SLURM_JOB_NAME")
        if not (user and name):
            return []
        listing = self.runner(["squeue", "-h", "-u", user, "-t", "PENDING", "-n", name, "-o", "%i"])
        out = [listing]
        if listing.get("returncode") == 0:
            out += [self.runner(["scontrol", "update", f"JobId={jid}", f"ExcNodeList={nodes_csv}"])
                    for jid in str(listing.get("stdout", "")).split()]
        return out

    def recover(self, bad_nodes: Sequence[str]) -> List[Dict[str, Any]]:
        if self.disabled or self.action == "exit":
            return []
        job = os.environ.get("SLURM_JOB_ID")
        if not job:
            return [{"cmd": "<slurm>", "returncode": None, "stderr": "SLURM_JOB_ID is not set"}]
        if not bad_nodes:
            return [{"cmd": "<slurm>", "returncode": None, "stderr": "no bad nodes reported"}]
        nodes_csv = ",".join(bad_nodes)
        if self.action == "requeue":
            return ([self.runner(["scontrol", "update", f"JobId={job}", f"ExcNodeList={nodes_csv}"])]
                    + self._exclude_from_pending_twins(nodes_csv) + [self.runner(["scontrol", "requeue", job])])
        return self._exclude_from_pending_twins(nodes_csv) + [self.runner(["scancel", job])]


# ----------------------------------------------------------------------------- watchdog


class _HealthLog:
    """JSONL files under ``<out_dir>/gpu_health``; with ``strict`` a write error propagates."""

    def __init__(self, out_dir: str, rank: int) -> None:
        self.root = Path(out_dir) / "gpu_health"
        self.rank = rank
        self.strict = False
        self.warned = False

    def directory(self) -> Path:
        self.root.mkdir(parents=True, exist_ok=True)
        return self.root

    def append(self, stem: str, payload: Dict[str, Any]) -> None:
        try:
            with (self.directory() / f"{stem}_rank{self.rank}.jsonl").open("a", encoding="utf-8") as fh:
                fh.write(json.dumps(payload, sort_keys=True) + "\n")
        except OSError as exc:
            if self.strict:
                raise
            if stem != "gpu_health_notices" and not self.warned:
                self.warned = True
                print(f"[gpu-health] failed to write {stem} log: {exc}", flush=True)


class GpuHealthWatchdog:
    """One GPU's readings and verdicts; also the base of the node-level background monitor."""

    def __init__(self, *, device: torch.device, out_dir: str, rank: int, world_size: int,
                 clock: Callable[[], float] = time.monotonic,
                 runner: Optional[Callable[[Sequence[str]], Dict[str, Any]]] = None) -> None:
        self.device = device
        self.out_dir = canonical_dir(out_dir)
        self.rank = int(rank)
        self.world_size = int(world_size)
        self.hostname = socket.gethostname()
        self.slurm_node = current_slurm_node()
        self.cuda_device = device.index if device.type == "cuda" and device.index is not None else None
        self.local_rank = current_local_rank()
        self.gpu_query_id = query_id_for_cuda_device(self.cuda_device)
        self.nvidia_smi = shutil.which("nvidia-smi")
        self.enabled = device.type == "cuda" and not _env_flag("KOOCHAK_GPU_HEALTH_DISABLE")
        self.slurm = SlurmRecovery.from_env(runner)
        self.exit_code = EXIT_CODE
        self.clock = clock
        self.verdicts = _Verdicts()
        self.log = _HealthLog(self.out_dir, self.rank)
        self._noticed = False

    # Slurm policy, as attributes of the watchdog.
    slurm_action = property(lambda self: self.slurm.action)
    requested_slurm_action = property(lambda self: self.slurm.requested_action)
    slurm_disabled = property(lambda self: self.slurm.disabled)
    slurm_mutation_blocked_reason = property(lambda self: self.slurm.blocked_reason)

    def should_check_step(self, step: int) -> bool:
        return self.enabled and step >= WARMUP_STEPS and step % CHECK_EVERY_STEPS == 0

    def check_local(self, step: int) -> Optional[GpuHealthFailure]:
        """Query this GPU and judge the reading; a missing reading ends any streak or heat episode."""

        sample = self.read_sample(step)
        if sample is None:
            self.verdicts.clear()
            return None
        return self.observe_sample(sample)

    def observe_sample(self, sample: GpuHealthSample) -> Optional[GpuHealthFailure]:
        reasons = evaluate_sample(sample, self.verdicts.thresholds)
        verdict, duration = self.verdicts.judge(reasons, self.clock())
        self.log.append("gpu_health", {**sample.to_dict(), "thermal_duration_seconds": duration,
                                       "thermal_grace_seconds": THERMAL_GRACE_SECONDS})
        if verdict is None:
            return None
        failed_reasons, count = verdict
        failure = GpuHealthFailure(sample=sample, reasons=failed_reasons, consecutive_failures=count,
                                   slurm_action=self.slurm_action, thermal_duration_seconds=duration)
        self.log.append("gpu_health_failures", failure.to_dict())
        return failure

    def read_sample(self, step: int) -> Optional[GpuHealthSample]:
        """One nvidia-smi query of this GPU (the fallback field list for older drivers)."""

        if self.nvidia_smi is None:
            self._notice("nvidia-smi is not available on PATH")
            return None
        for fields in (PRIMARY_QUERY_FIELDS, FALLBACK_QUERY_FIELDS):
            argv = [self.nvidia_smi, "-i", self.gpu_query_id, f"--query-gpu={','.join(fields)}",
                    "--format=csv,noheader,nounits"]
            try:
                done = subprocess.run(argv, check=False, capture_output=True, text=True, timeout=10.0)
            except (OSError, subprocess.SubprocessError) as exc:
                self._notice(f"nvidia-smi query failed: {exc}")
                return None
            if done.returncode == 0:
                sample = parse_nvidia_smi_csv(stdout=done.stdout, fields=fields, step=step, rank=self.rank,
                                              world_size=self.world_size, hostname=self.hostname,
                                              slurm_node=self.slurm_node, cuda_device=self.cuda_device,
                                              gpu_query_id=self.gpu_query_id)
                if sample is not None:
                    return sample
        self._notice("nvidia-smi did not return a parseable GPU health row")
        return None

    def gather_failures(self, local_failure: Optional[GpuHealthFailure]) -> List[Dict[str, Any]]:
        """Every rank's failure record (a collective when a process group exists)."""

        mine = None if local_failure is None else local_failure.to_dict()
        if not (torch.distributed.is_available() and torch.distributed.is_initialized()):
            return [] if mine is None else [mine]
        everyone: List[Optional[Dict[str, Any]]] = [None] * torch.distributed.get_world_size()
        torch.distributed.all_gather_object(everyone, mine)
        return [f for f in everyone if f is not None]

    def bad_nodes_from_failures(self, failures: Sequence[Dict[str, Any]]) -> List[str]:
        names = set()
        for f in failures:
            node = f.get("slurm_node")
            node = f.get("hostname") if not node or str(node).lower() == "unknown" else node
            if node:
                names.add(str(node))
        return self.slurm.node_names(sorted(names))

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
        target = self.log.directory() / f"gpu_health_failure_step{step:09d}.json"
        partial = target.with_name(target.name + ".tmp")
        partial.write_text(json.dumps(summary, indent=2, sort_keys=True) + "\n", encoding="utf-8")
        os.replace(partial, target)
        return str(target)

    def perform_slurm_recovery(self, failures: Sequence[Dict[str, Any]]) -> List[Dict[str, Any]]:
        if self.slurm.disabled or self.slurm.action == "exit":
            return []
        return self.slurm.recover(self.bad_nodes_from_failures(failures))

    def _notice(self, message: str) -> None:
        if self._noticed:
            return
        self._noticed = True
        self.log.append("gpu_health_notices", {
            "event": "gpu_health_notice", "rank": self.rank, "hostname": self.hostname,
            "slurm_node": self.slurm_node, "cuda_device": self.cuda_device, "gpu_query_id": self.gpu_query_id,
            "message": message, "timestamp_unix": time.time()})


def summarize_failures_for_stdout(failures: Iterable[Dict[str, Any]]) -> str:
    def one(f: Dict[str, Any]) -> str:
        return (f"rank={f.get('rank')} local_rank={f.get('local_rank')} host={f.get('hostname')} "
                f"node={f.get('slurm_node')} gpu={f.get('gpu_index')} uuid={f.get('gpu_uuid')} "
                f"reasons={','.join(str(r) for r in f.get('reasons', []))} temp={f.get('gpu_temp_c')}C "
                f"mem={f.get('memory_temp_c')}C sm={f.get('sm_clock_mhz')}/{f.get('max_sm_clock_mhz')}MHz "
                f"util={f.get('gpu_util_pct')}%")

    return " | ".join(one(f) for f in failures)
