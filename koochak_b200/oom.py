"""Opt-in recovery from CUDA out-of-memory errors inside a step (reference: koochak/oom.py:67-252).

Handled OOMs are those the caching allocator raises (``torch.OutOfMemoryError``)
while a step fetches micro-batches, runs ``step_fn`` or runs backward: before
any parameter, optimizer, EMA, scaler or scheduler state changes. The native
kernels allocate their outputs and scratch from the same allocator, so their
OOMs take this path too. Each handled step is recorded create-only under
``oom/`` in the checkpoint store before anything else happens, so a restarted
attempt skips it.
"""

from __future__ import annotations

import gc
import json
import re
from dataclasses import dataclass
from typing import AbstractSet, Any, Dict, FrozenSet, Optional

import torch

from .storage.store import Store
from .utils import config as config_lib

__all__ = ["FAIL", "OutOfMemoryError", "OomDecision", "OomRecoverySettings", "RECORD_PREFIX", "RESTART", "SKIP",
           "consecutive_run", "decide", "format_record", "memory_report", "record_key", "recorded_steps",
           "release_memory", "short_message", "write_record"]

OutOfMemoryError = torch.cuda.OutOfMemoryError
SKIP, RESTART, FAIL = "skip", "restart", "fail"
RECORD_PREFIX = "oom/"
_KEY = re.compile(r"oom/step(\d{9})-rank(\d{5})\.json")
_MAX_MESSAGE = 2000
_GIB = float(1 << 30)


def _positive(value: Any, label: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value < 1:
        raise ValueError(f"train.oom_recovery.{label} must be a positive integer, got {value!r}")
    return value


@dataclass(frozen=True)
class OomRecoverySettings:
    enabled: bool = False
    max_consecutive: int = 3
    max_skipped_steps: Optional[int] = None

    @classmethod
    def from_cfg(cls, train_cfg: Any) -> "OomRecoverySettings":
        cfg = config_lib.get(train_cfg, "oom_recovery", None)
        if cfg is None:
            return cls()
        cap = config_lib.get(cfg, "max_skipped_steps", None)
        return cls(enabled=bool(config_lib.get(cfg, "enabled", False)),
                   max_consecutive=_positive(config_lib.get(cfg, "max_consecutive", 3), "max_consecutive"),
                   max_skipped_steps=None if cap is None else _positive(cap, "max_skipped_steps"))


@dataclass(frozen=True)
class OomDecision:
    action: str
    consecutive: int
    skipped_total: int
    reason: str


def consecutive_run(skipped: AbstractSet[int], step: int) -> int:
    n = 1
    while step - n in skipped:
        n += 1
    return n


def decide(settings: OomRecoverySettings, skipped: AbstractSet[int], step: int, *, distributed: bool,
           during_fetch: bool) -> OomDecision:
    run = consecutive_run(skipped, step)
    total = len(skipped) + (0 if step in skipped else 1)
    if run > settings.max_consecutive:
        return OomDecision(FAIL, run, total, f"{run} consecutive OOM steps exceed "
                           f"train.oom_recovery.max_consecutive={settings.max_consecutive}")
    if settings.max_skipped_steps is not None and total > settings.max_skipped_steps:
        return OomDecision(FAIL, run, total, f"{total} OOM-skipped steps exceed "
                           f"train.oom_recovery.max_skipped_steps={settings.max_skipped_steps}")
    if distributed:
        return OomDecision(RESTART, run, total, "other ranks are blocked in this step's collectives")
    if during_fetch:
        return OomDecision(RESTART, run, total, "the data iterator may be unusable after an OOM inside it")
    if run == settings.max_consecutive:
        return OomDecision(RESTART, run, total, "a fresh process gets a fresh CUDA allocator")
    return OomDecision(SKIP, run, total, "skipped in place")


def record_key(step: int, rank: int) -> str:
    return f"{RECORD_PREFIX}step{int(step):09d}-rank{int(rank):05d}.json"


def recorded_steps(store: Store) -> FrozenSet[int]:
    found = set()
    for key in store.list(RECORD_PREFIX):
        m = _KEY.fullmatch(key)
        if m:
            found.add(int(m.group(1)))
    return frozenset(found)


def write_record(store: Store, record: Dict[str, Any]) -> str:
    key = record_key(record["step"], record["rank"])
    text = json.dumps(record, sort_keys=True, separators=(",", ":"), ensure_ascii=False) + "\n"
    try:
        store.put(key, text.encode("utf-8"))
    except FileExistsError:
        pass
    return key


def short_message(exc: BaseException) -> str:
    text = " ".join(str(exc).split())
    return text if len(text) <= _MAX_MESSAGE else text[: _MAX_MESSAGE - 3] + "..."


def memory_report(device: torch.device) -> tuple[Optional[Dict[str, int]], Optional[str]]:
    if getattr(device, "type", "cpu") != "cuda":
        return None, None
    free, total = torch.cuda.mem_get_info(device)
    stats = {
        "allocated_bytes": int(torch.cuda.memory_allocated(device)),
        "reserved_bytes": int(torch.cuda.memory_reserved(device)),
        "peak_allocated_bytes": int(torch.cuda.max_memory_allocated(device)),
        "free_bytes": int(free),
        "total_bytes": int(total),
    }
    return stats, torch.cuda.memory_summary(device, abbreviated=True)


def release_memory(device: torch.device) -> None:
    gc.collect()
    if getattr(device, "type", "cpu") == "cuda":
        torch.cuda.empty_cache()


def format_record(record: Dict[str, Any]) -> str:
    parts = [f"rank={record['rank']}", f"step={record['step']}", f"phase={record['phase']}",
             f"micro={record['micro_step'] + 1}/{record['grad_accum']}", f"action={record['action']}",
             f"consecutive={record['consecutive']}/{record['max_consecutive']}",
             f"skipped_total={record['skipped_total']}"]
    mem = record.get("memory")
    if mem:
        parts.append("allocated={:.2f}GiB reserved={:.2f}GiB peak={:.2f}GiB free={:.2f}GiB".format(
            mem["allocated_bytes"] / _GIB, mem["reserved_bytes"] / _GIB, mem["peak_allocated_bytes"] / _GIB,
            mem["free_bytes"] / _GIB))
    msg = str(record.get("message", ""))
    if len(msg) > 300:
        msg = msg[:297] + "..."
    return "[oom] " + " ".join(parts) + f" ({record['reason']}): {msg}"
