"""The ``train.*`` settings a run reads once, from a declarative key table.

(the keys and defaults of reference koochak/loop.py:167-423 and
koochak/config.py:68-127 -- an interface: existing YAML files must load)

``LoopSettings.from_cfg`` walks ``_KEYS`` -- (config key, attribute,
converter, default) -- instead of spelling every field out; the few keys with
cross-checks (bucket caps, directories) are resolved afterwards. EMA settings
come from the nested ``train.ema`` section, falling back to the legacy flat
``train.ema_*`` keys.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Mapping, Optional, Tuple

from ..utils import config as config_lib
from ..utils.paths import canonical_dir

__all__ = ["LoopSettings", "EmaSettings", "DualEmaSettings", "shard_mode"]


def _keys(cfg: Any) -> Callable[[str, Any], Any]:
    return lambda key, default=None: config_lib.get(cfg, key, default)


def _str_tuple(v: Any) -> Tuple[str, ...]:
    return tuple(str(x) for x in (v or ()))


# (config key, attribute, converter, default)
_KEYS: Tuple[Tuple[str, str, Callable[[Any], Any], Any], ...] = (
    ("ddp", "ddp_enabled", bool, False),
    ("shard_dataset", "shard_dataset_enabled", bool, False),
    ("shard_dataset_mode", "shard_dataset_mode", lambda v: v, None),
    ("shard_eval_dataset", "shard_eval_dataset_enabled", bool, False),
    ("shard_eval_dataset_mode", "shard_eval_dataset_mode", lambda v: v, None),
    ("warn_unsharded", "warn_unsharded", bool, True),
    ("amp", "amp_mode", str, "fp32"),
    ("grad_accum", "grad_accum", int, 1),
    ("grad_clip_norm", "grad_clip_norm", lambda v: v, None),
    ("nonfinite_grad_check_every", "nonfinite_grad_check_every", int, 0),
    ("scheduler_step", "scheduler_step_policy", str, "step"),
    ("max_steps", "max_steps", int, 100_000),
    ("log_every", "log_every", int, 100),
    ("eval_every", "eval_every", int, 5_000),
    ("eval_at_step_zero", "eval_at_step_zero", bool, True),
    ("ckpt_every", "ckpt_every", int, 5_000),
    ("intervals_use_completed_steps", "intervals_use_completed_steps", bool, False),
    ("rank_timing_every", "rank_timing_every", int, 0),
    ("rank_timing_keys", "rank_timing_extra_keys", _str_tuple, ()),
    ("keep_last_k", "keep_last_k", int, 3),
    ("checkpoint_async", "checkpoint_async", bool, False),
    ("prefetch_batches", "prefetch_batches", int, 0),
    ("prefetch_pipeline", "prefetch_pipeline", str, "single"),
    ("prefetch_threaded", "prefetch_threaded", bool, False),
    ("autocast_in_step_fn", "autocast_in_step_fn", bool, False),
    ("scalarize_loss_every_step", "scalarize_loss_every_step", bool, True),
    ("profile_step_fn_timing", "profile_step_timing", bool, False),
    ("profile_step_fn_cuda_sync", "profile_step_cuda_sync", bool, True),
    ("find_unused_parameters", "find_unused_parameters", bool, False),
    ("ddp_static_graph", "ddp_static_graph", bool, False),
    ("ddp_gradient_as_bucket_view", "ddp_gradient_as_bucket_view", bool, False),
    ("ddp_broadcast_buffers", "ddp_broadcast_buffers", bool, True),
    ("device_timing", "device_timing", bool, False),
    ("comm_transport", "comm_transport", str, "auto"),
    ("profile_nvtx", "profile_nvtx", bool, False),
    ("cuda_graph_step", "cuda_graph_step", bool, False),
    ("cuda_graph_warmup", "cuda_graph_warmup", int, 3),
)


@dataclass
class LoopSettings:
    ddp_enabled: bool = False
    shard_dataset_enabled: bool = False
    shard_dataset_mode: Optional[str] = None
    shard_eval_dataset_enabled: bool = False
    shard_eval_dataset_mode: Optional[str] = None
    warn_unsharded: bool = True
    amp_mode: str = "fp32"
    grad_accum: int = 1
    grad_clip_norm: Optional[float] = None
    nonfinite_grad_check_every: int = 0
    scheduler_step_policy: str = "step"
    max_steps: int = 100_000
    log_every: int = 100
    eval_every: int = 5_000
    eval_at_step_zero: bool = True
    ckpt_every: int = 5_000
    intervals_use_completed_steps: bool = False
    rank_timing_every: int = 0
    rank_timing_extra_keys: Tuple[str, ...] = ()
    out_dir: str = ""
    keep_last_k: int = 3
    checkpoint_dir: str = ""
    checkpoint_async: bool = False
    prefetch_batches: int = 0
    prefetch_pipeline: str = "single"
    prefetch_threaded: bool = False
    autocast_in_step_fn: bool = False
    scalarize_loss_every_step: bool = True
    profile_step_timing: bool = False
    profile_step_cuda_sync: bool = True
    find_unused_parameters: bool = False
    ddp_static_graph: bool = False
    ddp_gradient_as_bucket_view: bool = False
    ddp_bucket_cap_mb: Optional[int] = None
    ddp_bucket_cap_mb_list: Optional[Tuple[int, ...]] = None
    ddp_broadcast_buffers: bool = True
    device_timing: bool = False
    comm_transport: str = "auto"
    profile_nvtx: bool = False
    cuda_graph_step: bool = False
    cuda_graph_warmup: int = 3

    @classmethod
    def from_cfg(cls, cfg: Any) -> "LoopSettings":
        get = _keys(cfg)
        values: Dict[str, Any] = {}
        for key, attr, convert, default in _KEYS:
            raw = get(key, default)
            values[attr] = default if raw is None and default is None else convert(raw)
        cap, caps = get("ddp_bucket_cap_mb", None), get("ddp_bucket_cap_mb_list", None)
        if cap is not None and caps is not None:
            raise ValueError("Set only one of train.ddp_bucket_cap_mb and train.ddp_bucket_cap_mb_list")
        if caps is not None:
            caps = tuple(int(v) for v in caps)
            if not caps or min(caps) <= 0:
                raise ValueError("train.ddp_bucket_cap_mb_list must contain positive values")
        values["ddp_bucket_cap_mb"] = None if cap is None else int(cap)
        values["ddp_bucket_cap_mb_list"] = caps
        out = canonical_dir(get("out_dir", "./runs/exp0"))
        where = get("checkpoint_dir", None)
        values["out_dir"] = out
        values["checkpoint_dir"] = out if where is None else (str(where) if "://" in str(where)
                                                              else canonical_dir(where))
        return cls(**values)

    def bucket_caps_mb(self) -> list:
        """Gradient bucket sizes in MB (a single cap is a one-entry list; torch DDP's 25 MB by default)."""

        if self.ddp_bucket_cap_mb is not None:
            return [float(self.ddp_bucket_cap_mb)]
        return [float(c) for c in (self.ddp_bucket_cap_mb_list or (25,))]


def shard_mode(enabled: bool, mode: Any, label: str) -> Optional[str]:
    """The validated sharding mode of ``train.<label>`` (None when sharding is off)."""

    if not enabled:
        return None
    if mode is None:
        raise ValueError(f"train.{label}_mode must be set when train.{label}=true")
    if str(mode).lower() not in ("iterable", "map"):
        raise ValueError(f"Invalid train.{label}_mode: {mode!r} (expected 'iterable' or 'map')")
    return str(mode).lower()


# Legacy flat keys: train.ema_<x> for train.ema.<x>.
_FLAT = {"enabled": "ema_enabled", "decay": "ema_decay", "decay_init": "ema_decay_init",
         "warmup_steps": "ema_warmup_steps", "schedule": "ema_schedule", "profile": "ema_profile",
         "gamma": "ema_gamma", "srel": "ema_srel", "offload_to_cpu": "ema_offload_to_cpu",
         "pin_memory": "ema_pin_memory", "update_every": "ema_update_every",
         "compensate_update_every": "ema_compensate_update_every", "eval_with_ema": "ema_eval"}
_RAMPS = frozenset({"linear", "ramp", "warmup", "cosine"})


def _ema_reader(train_cfg: Any) -> Callable[[str, Any], Any]:
    section = config_lib.get(train_cfg, "ema", {}) if train_cfg is not None else {}

    def read(key: str, default: Any = None) -> Any:
        if isinstance(section, Mapping):
            nested = config_lib.get(section, key, None) if key in section else None
        else:
            nested = getattr(section, key, None)
        if nested is not None:
            return nested
        if key not in _FLAT:
            return default
        flat = config_lib.get(train_cfg, _FLAT[key], default)
        return default if flat is None else flat

    return read


@dataclass
class DualEmaSettings:
    enabled: bool = False
    gamma1: Optional[float] = None
    gamma2: Optional[float] = None
    srel1: Optional[float] = None
    srel2: Optional[float] = None

    @classmethod
    def from_cfg(cls, ema_cfg: Any) -> "DualEmaSettings":
        dual = config_lib.get(ema_cfg, "dual", {}) if ema_cfg is not None else {}
        get = _keys(dual)
        return cls(bool(get("enabled", False)), get("gamma1"), get("gamma2"), get("srel1"), get("srel2"))


@dataclass
class EmaSettings:
    enabled: bool = False
    profile: str = "constant"
    target_decay: Optional[float] = None
    decay_init: Optional[float] = None
    warmup_steps: int = 0
    schedule: str = "constant"
    gamma: Optional[float] = None
    srel: Optional[float] = None
    offload_to_cpu: bool = True
    pin_memory: bool = True
    update_every: int = 1
    compensate_update_every: bool = True
    eval_with_ema: bool = False
    dual: DualEmaSettings = field(default_factory=DualEmaSettings)

    @classmethod
    def from_cfg(cls, train_cfg: Any) -> "EmaSettings":
        read = _ema_reader(train_cfg)
        switch = read("enabled", None)
        if switch is None:  # no explicit switch: a decay or a non-constant profile turns it on
            profile = read("profile", None)
            on = read("decay", None) is not None or (
                profile is not None and str(profile).lower() not in ("", "none", "constant"))
        else:
            on = bool(switch)
        section = config_lib.get(train_cfg, "ema", {}) if train_cfg is not None else {}
        common = dict(gamma=read("gamma"), srel=read("srel"), offload_to_cpu=bool(read("offload_to_cpu", True)),
                      pin_memory=bool(read("pin_memory", True)), update_every=max(1, int(read("update_every", 1))),
                      compensate_update_every=bool(read("compensate_update_every", True)),
                      dual=DualEmaSettings.from_cfg(section))
        if not on:
            return cls(**common)
        target = float(read("decay", 0.999))
        return cls(enabled=True, profile=str(read("profile", "constant")).lower(), target_decay=target,
                   decay_init=float(read("decay_init", min(0.9, target))), warmup_steps=int(read("warmup_steps", 0)),
                   schedule=str(read("schedule", "constant")).lower(), eval_with_ema=bool(read("eval_with_ema", False)),
                   **common)

    def warmed_decay(self, step: int) -> float:
        """The constant-profile decay at ``step`` (ramped from ``decay_init`` over ``warmup_steps``)."""

        target = float(self.target_decay or 0.999)
        if self.warmup_steps <= 0 or self.schedule not in _RAMPS:
            return target
        progress = min(1.0, max(0.0, (step + 1) / float(self.warmup_steps)))
        if self.schedule == "cosine":
            progress = 0.5 * (1.0 - math.cos(math.pi * progress))
        start = self.decay_init or target
        return float(min(max(start + (target - start) * progress, 0.0), 0.999999))
