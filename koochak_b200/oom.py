"""Surviving CUDA out-of-memory errors inside a training step (opt-in).

(behaviour of reference koochak/oom.py:67-252)

An OOM is recoverable when the caching allocator raises it
(``torch.OutOfMemoryError``) while a step fetches micro-batches, runs
``step_fn`` or runs backward -- before any parameter, optimizer, EMA, scaler
or scheduler state has changed. This library's kernels allocate outputs and
scratch from the same allocator, so their OOMs take the same route.

What happens to such a step is decided by ``decide``: an ordered list of
rules, the first that matches wins --

1. too many consecutive OOM steps            -> fail
2. too many OOM-skipped steps in total        -> fail
3. other ranks exist (they wait in this step's collectives) -> restart
4. the OOM came from the data iterator (it may be unusable) -> restart
5. this is the last consecutive OOM allowed (a fresh process gets a fresh
   allocator)                                 -> restart
6. otherwise                                  -> skip the step in place.

Every handled step is recorded create-only in the checkpoint store, as
``oom/step<9 digits>-rank<5 digits>.json`` (a format shared with the
reference), before anything else can fail, so a restarted attempt knows to
skip it.
"""

from __future__ import annotations

import gc
import json
import re
from dataclasses import dataclass
from typing import AbstractSet, Any, Callable, Dict, FrozenSet, List, Optional, Tuple

import torch

from .storage.store import Store
from .utils import config as config_lib

__all__ = ["FAIL", "OutOfMemoryError", "OomDecision", "OomRecoverySettings", "RECORD_PREFIX", "RESTART", "SKIP",
           "consecutive_run", "decide", "format_record", "memory_report", "record_key", "recorded_steps",
           "release_memory", "short_message", "write_record"]

OutOfMemoryError = torch.cuda.OutOfMemoryError
SKIP, RESTART, FAIL = "skip", "restart", "fail"
RECORD_PREFIX = "oom/"
_RECORD_NAME = re.compile(r"oom/step(?P<step>\d{9})-rank(?P<rank>\d{5})\.json")
_MESSAGE_LIMIT = 2000
_LOG_MESSAGE_LIMIT = 300
_GIB = float(1 << 30)


def _positive_int(value: Any, key: str) -> int:
    ok = isinstance(value, int) and not isinstance(value, bool) and value >= 1
    if not ok:
        raise ValueError(f"train.oom_recovery.{key} must be a positive integer, got {value!r}")
    return value


@dataclass(frozen=True)
class OomRecoverySettings:
    enabled: bool = False
    max_consecutive: int = 3
    max_skipped_steps: Optional[int] = None

    @classmethod
    def from_cfg(cls, train_cfg: Any) -> "OomRecoverySettings":
        section = config_lib.get(train_cfg, "oom_recovery", None)
        if section is None:
            return cls()
        read = lambda key, default: config_lib.get(section, key, default)  # noqa: E731
        cap = read("max_skipped_steps", None)
        return cls(enabled=bool(read("enabled", False)),
                   max_consecutive=_positive_int(read("max_consecutive", 3), "max_consecutive"),
                   max_skipped_steps=None if cap is None else _positive_int(cap, "max_skipped_steps"))


@dataclass(frozen=True)
class OomDecision:
    action: str
    consecutive: int
    skipped_total: int
    reason: str


def consecutive_run(skipped: AbstractSet[int], step: int) -> int:
    """Length of the run of OOM steps that ends at ``step`` (``step`` itself included)."""

    start = step
    while start - 1 in skipped:
        start -= 1
    return step - start + 1


@dataclass(frozen=True)
class _Situation:
    settings: OomRecoverySettings
    run: int
    total: int
    distributed: bool
    during_fetch: bool


_Rule = Tuple[Callable[[_Situation], bool], str, Callable[[_Situation], str]]

_RULES: List[_Rule] = [
    (lambda s: s.run > s.settings.max_consecutive, FAIL,
     lambda s: f"{s.run} consecutive OOM steps exceed train.oom_recovery.max_consecutive={s.settings.max_consecutive}"),
    (lambda s: s.settings.max_skipped_steps is not None and s.total > s.settings.max_skipped_steps, FAIL,
     lambda s: f"{s.total} OOM-skipped steps exceed "
               f"train.oom_recovery.max_skipped_steps={s.settings.max_skipped_steps}"),
    (lambda s: s.distributed, RESTART, lambda s: "other ranks are blocked in this step's collectives"),
    (lambda s: s.during_fetch, RESTART, lambda s: "the data iterator may be unusable after an OOM inside it"),
    (lambda s: s.run == s.settings.max_consecutive, RESTART, lambda s: "a fresh process gets a fresh CUDA allocator"),
    (lambda s: True, SKIP, lambda s: "skipped in place"),
]


def decide(settings: OomRecoverySettings, skipped: AbstractSet[int], step: int, *, distributed: bool,
           during_fetch: bool) -> OomDecision:
    """What to do with an OOM at ``step``, given the steps already skipped for OOM."""

    situation = _Situation(settings, consecutive_run(skipped, step), len(skipped | {step}), distributed, during_fetch)
    for matches, action, why in _RULES:
        if matches(situation):
            return OomDecision(action, situation.run, situation.total, why(situation))
    raise AssertionError("unreachable: the last rule always matches")


def record_key(step: int, rank: int) -> str:
    return f"{RECORD_PREFIX}step{int(step):09d}-rank{int(rank):05d}.json"


def recorded_steps(store: Store) -> FrozenSet[int]:
    """Steps for which any rank left an OOM record."""

    hits = (_RECORD_NAME.fullmatch(k) for k in store.list(RECORD_PREFIX))
    return frozenset(int(m.group("step")) for m in hits if m is not None)


def write_record(store: Store, record: Dict[str, Any]) -> str:
    """Store ``record`` create-only (an existing record of the same step and rank is kept)."""

    key = record_key(record["step"], record["rank"])
    payload = json.dumps(record, sort_keys=True, separators=(",", ":"), ensure_ascii=False) + "\n"
    try:
        store.put(key, payload.encode("utf-8"))
    except FileExistsError:
        pass
    return key


def _clip(text: str, limit: int) -> str:
    return text if len(text) <= limit else text[: limit - 3] + "..."


def short_message(exc: BaseException) -> str:
    """The exception text on one line, at most 2000 characters."""

    return _clip(" ".join(str(exc).split()), _MESSAGE_LIMIT)


def memory_report(device: torch.device) -> Tuple[Optional[Dict[str, int]], Optional[str]]:
    """Allocator figures and the abbreviated allocator summary of a CUDA device (``None`` elsewhere)."""

    if getattr(device, "type", "cpu") != "cuda":
        return None, None
    free, total = torch.cuda.mem_get_info(device)
    figures = {
        "allocated_bytes": torch.cuda.memory_allocated(device),
        "reserved_bytes": torch.cuda.memory_reserved(device),
        "peak_allocated_bytes": torch.cuda.max_memory_allocated(device),
        "free_bytes": free,
        "total_bytes": total,
    }
    return {k: int(v) for k, v in figures.items()}, torch.cuda.memory_summary(device, abbreviated=True)


def release_memory(device: torch.device) -> None:
    """Drop Python garbage and return cached blocks so the next attempt starts from a lean allocator."""

    gc.collect()
    if getattr(device, "type", "cpu") == "cuda":
        torch.cuda.empty_cache()


def format_record(record: Dict[str, Any]) -> str:
    """One log line for an OOM record."""

    fields = [
        ("rank", record["rank"]), ("step", record["step"]), ("phase", record["phase"]),
        ("micro", f"{record['micro_step'] + 1}/{record['grad_accum']}"), ("action", record["action"]),
        ("consecutive", f"{record['consecutive']}/{record['max_consecutive']}"),
        ("skipped_total", record["skipped_total"]),
    ]
    words = [f"{k}={v}" for k, v in fields]
    mem = record.get("memory")
    if mem:
        gib = {k: mem[f"{k}_bytes"] / _GIB for k in ("allocated", "reserved", "peak_allocated", "free")}
        words.append("allocated={allocated:.2f}GiB reserved={reserved:.2f}GiB peak={peak_allocated:.2f}GiB "
                     "free={free:.2f}GiB".format(**gib))
    message = _clip(str(record.get("message", "")), _LOG_MESSAGE_LIMIT)
    return "[oom] " + " ".join(words) + f" ({record['reason']}): {message}"
