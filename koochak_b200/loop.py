"""``training_loop``: the function-first training runtime (reference: koochak/loop.py:437-1739).

The public contract matches the reference: the caller supplies a model, a
dataset, ``step_fn(model, batch, ctx) -> {"loss": tensor, ...}``, an
optimizer and a ``train`` config; the loop owns micro-batching and gradient
accumulation, AMP and the GradScaler, the gradient gate (unscale, finite
check, clipping), the optimizer/EMA/scheduler update, data parallelism, hooks
and logging, periodic/async/terminal checkpoints in the published ``.pt`` +
``.ready.json`` format, auto-resume, OOM skip/restart, SIGUSR1 evacuation and
the background GPU-health watchdog.

What runs differently on CUDA:

* gradient gate: one native pass computes the finite flag, per-tensor norms
  and the clip coefficient (and unscales for fp16); the host reads three
  numbers once; fused optimizers apply the coefficient when they read the
  gradients;
* update: optimizers from this package fuse the GPU-resident EMA into their
  parameter-update kernels;
* data parallelism (``ddp: true``): :class:`koochak_b200.parallel.ddp.DataParallel`
  with bucketed reductions overlapped with backward (NCCL, or the native
  P2P path with ``comm.transport: p2p``);
* optional device timing (``device_timing: true``): CUDA events bracket every
  update; ``on_update_end`` logs carry ``step_device_ms``.
"""

from __future__ import annotations

import json
import math
import os
import statistics
import time
import warnings
from contextlib import ExitStack, nullcontext
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterable, Iterator, Mapping, Optional, Sequence

import torch
import torch.nn as nn
from torch.amp import GradScaler
from torch.optim import Optimizer
from torch.optim.lr_scheduler import _LRScheduler

from . import oom as oom_lib
from .core import dist as dist_lib
from .core import hooks as hooks_lib
from .core.precision import Scaler as make_scaler
from .core.precision import FusedGradScaler, autocast_context, prepare_compile_backend
from .data.iterable import prefetch, to_device
from .data.sharding import shard_dataset, warn_if_unsharded
from .health.background import BackgroundGpuHealth
from .health.gpu import summarize_failures_for_stdout
from .interruption import EVACUATION_EXIT_CODE, OOM_RESTART_EXIT_CODE, EvacuationController
from .optim.grad_clip import GradientClipStats, clip_grad_norm_, fused_grad_gate
from .storage import checkpoint as checkpoint_lib
from .utils import config as config_lib
from .utils import flags as flags_lib
from .utils.collector import WarmFreeze
from .utils.device import ensure_process_device, get_device, get_lr
from .utils.ema import EMA
from .utils.paths import canonical_dir
from .utils.seed import get_rng_state, set_rng_state

__all__ = ["training_loop", "StepFn", "EvalFn", "BatchPrepareFn"]

StepFn = Callable[[nn.Module, Any, Mapping[str, Any]], Dict[str, Any]]
EvalFn = Callable[[nn.Module, Iterable, Mapping[str, Any]], Dict[str, float]]
BatchPrepareFn = Callable[[Any], Any]

_TIMING_KEYS = ("batch_wait_s", "step_compute_s", "total_step_s")
_ROOT_SIBLINGS = ("data", "optim", "logging", "wandb", "entry")
_EMA_FLAT_KEYS = {
    "enabled": "ema_enabled", "decay": "ema_decay", "decay_init": "ema_decay_init",
    "warmup_steps": "ema_warmup_steps", "schedule": "ema_schedule", "profile": "ema_profile",
    "gamma": "ema_gamma", "srel": "ema_srel", "offload_to_cpu": "ema_offload_to_cpu",
    "pin_memory": "ema_pin_memory", "update_every": "ema_update_every",
    "compensate_update_every": "ema_compensate_update_every", "eval_with_ema": "ema_eval",
}
_EMA_RAMPS = frozenset({"linear", "ramp", "warmup", "cosine"})
_WRAPS_ONLY = frozenset({"wraps", "wraps-only", "merge-wraps", "merge_wraps"})
_FULL = frozenset({"full", "full-model", "full_model"})


def _emit(hooks, event: str, *args, suppress_exceptions: bool = True, **kwargs) -> None:
    hooks_lib.emit(hooks, event, *args, suppress_exceptions=suppress_exceptions, **kwargs)


def _parameter_counts(module: nn.Module) -> Dict[str, int]:
    base = getattr(module, "module", module)
    total = sum(p.numel() for p in base.parameters())
    trainable = sum(p.numel() for p in base.parameters() if p.requires_grad)
    return {"total": int(total), "trainable": int(trainable), "frozen": int(total - trainable)}


def _batch_total(batch: Any, key: str) -> float:
    if not isinstance(batch, Mapping) or key not in batch:
        return 0.0
    v = batch[key]
    if isinstance(v, torch.Tensor):
        return float(v.detach().to(torch.float32).sum().item())
    if isinstance(v, (list, tuple)):
        return float(sum(float(x) for x in v)) if v else 0.0
    return float(v)


def _skip_counts(batch: Any) -> Dict[str, float]:
    if not isinstance(batch, Mapping):
        return {}
    return {str(k): _batch_total(batch, str(k)) for k in batch.keys() if str(k).endswith("_skip_count")}


def _timing_fragment(entries: list, key: str) -> str:
    if not entries:
        return f"{key}=n/a"
    ordered = sorted((float(e.get(key, 0.0)), int(e.get("rank", 0))) for e in entries)
    vals = [v for v, _ in ordered]
    slow, slow_rank = ordered[-1]
    return (f"{key}={ordered[0][0]:.3f}/{statistics.median(vals):.3f}/{slow:.3f}@r{slow_rank} "
            f"span={slow - ordered[0][0]:.3f}")


def _format_rank_timing(entries: list, step: int, extra_keys: Sequence[str] = ()) -> str:
    return f"[rank-timing] step={step} " + " ".join(_timing_fragment(entries, k) for k in (*_TIMING_KEYS, *extra_keys))


def _looks_like_root_config(cfg: Any) -> bool:
    if isinstance(cfg, Mapping):
        return "train" in cfg and any(k in cfg for k in _ROOT_SIBLINGS)
    return all(hasattr(cfg, k) for k in ("train",) + _ROOT_SIBLINGS)


def _resolve_train_config(train_cfg: Any, config_json: Optional[Mapping[str, Any]]):
    if _looks_like_root_config(train_cfg):
        warnings.warn("training_loop now expects train_cfg only; passing the full root config is deprecated.",
                      DeprecationWarning)
        config_json = config_json or train_cfg
        train_cfg = config_lib.get(train_cfg, "train", {})
    return train_cfg or {}, config_json


def _shard_mode(enabled: bool, mode: Any, label: str) -> Optional[str]:
    if not enabled:
        return None
    if mode is None:
        raise ValueError(f"train.{label}_mode must be set when train.{label}=true")
    key = str(mode).lower()
    if key not in ("iterable", "map"):
        raise ValueError(f"Invalid train.{label}_mode: {mode!r} (expected 'iterable' or 'map')")
    return key


@dataclass
class _TrainSettings:
    ddp_enabled: bool
    shard_dataset_enabled: bool
    shard_dataset_mode: Optional[str]
    shard_eval_dataset_enabled: bool
    shard_eval_dataset_mode: Optional[str]
    warn_unsharded: bool
    amp_mode: str
    grad_accum: int
    grad_clip_norm: Optional[float]
    nonfinite_grad_check_every: int
    scheduler_step_policy: str
    max_steps: int
    log_every: int
    eval_every: int
    eval_at_step_zero: bool
    ckpt_every: int
    intervals_use_completed_steps: bool
    rank_timing_every: int
    rank_timing_extra_keys: tuple
    out_dir: str
    keep_last_k: int
    checkpoint_dir: str
    checkpoint_async: bool
    prefetch_batches: int
    prefetch_pipeline: str
    prefetch_threaded: bool
    autocast_in_step_fn: bool
    scalarize_loss_every_step: bool
    profile_step_timing: bool
    profile_step_cuda_sync: bool
    find_unused_parameters: bool
    ddp_static_graph: bool
    ddp_gradient_as_bucket_view: bool
    ddp_bucket_cap_mb: Optional[int]
    ddp_bucket_cap_mb_list: Optional[tuple]
    ddp_broadcast_buffers: bool
    device_timing: bool = False
    comm_transport: str = "auto"
    profile_nvtx: bool = False

    @classmethod
    def from_cfg(cls, cfg: Any) -> "_TrainSettings":
        g = config_lib.get
        cap, cap_list = g(cfg, "ddp_bucket_cap_mb", None), g(cfg, "ddp_bucket_cap_mb_list", None)
        if cap is not None and cap_list is not None:
            raise ValueError("Set only one of train.ddp_bucket_cap_mb and train.ddp_bucket_cap_mb_list")
        caps = tuple(int(v) for v in cap_list) if cap_list is not None else None
        if caps is not None and (not caps or any(v <= 0 for v in caps)):
            raise ValueError("train.ddp_bucket_cap_mb_list must contain positive values")
        out_dir = canonical_dir(g(cfg, "out_dir", "./runs/exp0"))
        ckpt_dir = g(cfg, "checkpoint_dir", None)
        if ckpt_dir is None:
            ckpt_dir = out_dir
        elif "://" not in str(ckpt_dir):
            ckpt_dir = canonical_dir(ckpt_dir)
        return cls(
            ddp_enabled=bool(g(cfg, "ddp", False)),
            shard_dataset_enabled=bool(g(cfg, "shard_dataset", False)),
            shard_dataset_mode=g(cfg, "shard_dataset_mode", None),
            shard_eval_dataset_enabled=bool(g(cfg, "shard_eval_dataset", False)),
            shard_eval_dataset_mode=g(cfg, "shard_eval_dataset_mode", None),
            warn_unsharded=bool(g(cfg, "warn_unsharded", True)),
            amp_mode=str(g(cfg, "amp", "fp32")),
            grad_accum=int(g(cfg, "grad_accum", 1)),
            grad_clip_norm=g(cfg, "grad_clip_norm", None),
            nonfinite_grad_check_every=int(g(cfg, "nonfinite_grad_check_every", 0)),
            scheduler_step_policy=str(g(cfg, "scheduler_step", "step")),
            max_steps=int(g(cfg, "max_steps", 100_000)),
            log_every=int(g(cfg, "log_every", 100)),
            eval_every=int(g(cfg, "eval_every", 5_000)),
            eval_at_step_zero=bool(g(cfg, "eval_at_step_zero", True)),
            ckpt_every=int(g(cfg, "ckpt_every", 5_000)),
            intervals_use_completed_steps=bool(g(cfg, "intervals_use_completed_steps", False)),
            rank_timing_every=int(g(cfg, "rank_timing_every", 0)),
            rank_timing_extra_keys=tuple(str(k) for k in (g(cfg, "rank_timing_keys", ()) or ())),
            out_dir=out_dir,
            keep_last_k=int(g(cfg, "keep_last_k", 3)),
            checkpoint_dir=str(ckpt_dir),
            checkpoint_async=bool(g(cfg, "checkpoint_async", False)),
            prefetch_batches=int(g(cfg, "prefetch_batches", 0)),
            prefetch_pipeline=str(g(cfg, "prefetch_pipeline", "single")),
            prefetch_threaded=bool(g(cfg, "prefetch_threaded", False)),
            autocast_in_step_fn=bool(g(cfg, "autocast_in_step_fn", False)),
            scalarize_loss_every_step=bool(g(cfg, "scalarize_loss_every_step", True)),
            profile_step_timing=bool(g(cfg, "profile_step_fn_timing", False)),
            profile_step_cuda_sync=bool(g(cfg, "profile_step_fn_cuda_sync", True)),
            find_unused_parameters=bool(g(cfg, "find_unused_parameters", False)),
            ddp_static_graph=bool(g(cfg, "ddp_static_graph", False)),
            ddp_gradient_as_bucket_view=bool(g(cfg, "ddp_gradient_as_bucket_view", False)),
            ddp_bucket_cap_mb=int(cap) if cap is not None else None,
            ddp_bucket_cap_mb_list=caps,
            ddp_broadcast_buffers=bool(g(cfg, "ddp_broadcast_buffers", True)),
            device_timing=bool(g(cfg, "device_timing", False)),
            comm_transport=str(g(cfg, "comm_transport", "auto")),
            profile_nvtx=bool(g(cfg, "profile_nvtx", False)),
        )


@dataclass
class _DualEmaSettings:
    enabled: bool
    gamma1: Optional[float]
    gamma2: Optional[float]
    srel1: Optional[float]
    srel2: Optional[float]

    @classmethod
    def from_cfg(cls, ema_cfg: Any) -> "_DualEmaSettings":
        d = config_lib.get(ema_cfg, "dual", {}) if ema_cfg is not None else {}
        g = config_lib.get
        return cls(bool(g(d, "enabled", False)), g(d, "gamma1", None), g(d, "gamma2", None), g(d, "srel1", None),
                   g(d, "srel2", None))


def _ema_getter(train_cfg: Any) -> Callable[[str, Any], Any]:
    """Read ``train.ema.<key>``, falling back to the legacy flat ``train.ema_<key>``."""

    ema_cfg = config_lib.get(train_cfg, "ema", {}) if train_cfg is not None else {}

    def get(key: str, default: Any = None) -> Any:
        if isinstance(ema_cfg, Mapping):
            if key in ema_cfg:
                v = config_lib.get(ema_cfg, key, default)
                if v is not None:
                    return v
        else:
            v = getattr(ema_cfg, key, None)
            if v is not None:
                return v
        flat = _EMA_FLAT_KEYS.get(key)
        if flat is None:
            return default
        v = config_lib.get(train_cfg, flat, default)
        return default if v is None else v

    return get


@dataclass
class _EmaSettings:
    enabled: bool
    profile: str
    target_decay: Optional[float]
    decay_init: Optional[float]
    warmup_steps: int
    schedule: str
    gamma: Optional[float]
    srel: Optional[float]
    offload_to_cpu: bool
    pin_memory: bool
    update_every: int
    compensate_update_every: bool
    eval_with_ema: bool
    dual: _DualEmaSettings

    @classmethod
    def from_cfg(cls, train_cfg: Any) -> "_EmaSettings":
        get = _ema_getter(train_cfg)
        ema_cfg = config_lib.get(train_cfg, "ema", {}) if train_cfg is not None else {}
        flag = get("enabled", None)
        if flag is None:
            prof = get("profile", None)
            enabled = get("decay", None) is not None or (prof is not None and str(prof).lower()
                                                          not in ("", "none", "constant"))
        else:
            enabled = bool(flag)
        target = float(get("decay", 0.999)) if enabled else None
        return cls(
            enabled=enabled,
            profile=str(get("profile", "constant")).lower() if enabled else "constant",
            target_decay=target,
            decay_init=float(get("decay_init", min(0.9, target or 0.999))) if enabled else None,
            warmup_steps=int(get("warmup_steps", 0)) if enabled else 0,
            schedule=str(get("schedule", "constant")).lower() if enabled else "constant",
            gamma=get("gamma", None),
            srel=get("srel", None),
            offload_to_cpu=bool(get("offload_to_cpu", True)),
            pin_memory=bool(get("pin_memory", True)),
            update_every=max(1, int(get("update_every", 1))),
            compensate_update_every=bool(get("compensate_update_every", True)),
            eval_with_ema=bool(get("eval_with_ema", False)) if enabled else False,
            dual=_DualEmaSettings.from_cfg(ema_cfg),
        )

    def warmed_decay(self, step: int) -> float:
        d = float(self.target_decay or 0.999)
        if self.warmup_steps <= 0 or self.schedule not in _EMA_RAMPS:
            return d
        t = max(0.0, min(1.0, (step + 1) / float(self.warmup_steps)))
        s = 0.5 * (1.0 - math.cos(math.pi * t)) if self.schedule == "cosine" else t
        init = self.decay_init or d
        return float(min(max(init + (d - init) * s, 0.0), 0.999999))

    def _make(self, module: nn.Module, profile: str, gamma, srel) -> EMA:
        return EMA(module, decay=float(self.target_decay or 0.999), profile=profile, gamma=gamma, srel=srel,
                   update_every=self.update_every, offload_to_cpu=self.offload_to_cpu, pin_memory=self.pin_memory,
                   compensate_update_every=self.compensate_update_every)

    def build(self, module: nn.Module) -> EMA:
        return self._make(module, self.profile, self.gamma, self.srel)

    def build_dual(self, module: nn.Module) -> list:
        if not self.dual.enabled:
            return []
        return [self._make(module, "power", self.dual.gamma1, self.dual.srel1),
                self._make(module, "power", self.dual.gamma2, self.dual.srel2)]


@dataclass
class _MicroStats:
    out: Optional[Dict[str, Any]] = None
    total_loss: Optional[torch.Tensor] = None
    total_loss_scalar: Optional[float] = None
    batch_wait_s: float = 0.0
    extra_timing_totals: Dict[str, float] = field(default_factory=dict)
    profile_timing_totals: Dict[str, float] = field(default_factory=dict)
    skip_count_totals: Dict[str, float] = field(default_factory=dict)


def training_loop(*, model: nn.Module, dataset: Iterable, step_fn: StepFn, optimizer: Optimizer,
                  scheduler: Optional[_LRScheduler] = None, train_cfg: Mapping[str, Any] | Any,
                  config_json: Optional[Mapping[str, Any]] = None, checkpoint_dict: Optional[Dict[str, Any]] = None,
                  eval_dataset: Optional[Iterable] = None, eval_fn: Optional[EvalFn] = None,
                  prepare_batch_fn: Optional[BatchPrepareFn] = None,
                  hooks: Optional[Dict[str, list[Callable]]] = None, resume: Optional[str] = None,
                  auto_resume_path: Optional[str] = None,
                  evacuation: Optional[EvacuationController | bool] = None) -> Dict[str, Any]:
    """Train until ``train.max_steps`` or dataset exhaustion; return the final checkpoint dict."""

    return _TrainLoop(model=model, dataset=dataset, step_fn=step_fn, optimizer=optimizer, scheduler=scheduler,
                      train_cfg=train_cfg, config_json=config_json, checkpoint_dict=checkpoint_dict,
                      eval_dataset=eval_dataset, eval_fn=eval_fn, prepare_batch_fn=prepare_batch_fn, hooks=hooks,
                      resume=resume, auto_resume_path=auto_resume_path, evacuation=evacuation).run()


class _TrainLoop:
    """Orchestrator behind ``training_loop`` (not public API)."""

    def __init__(self, *, model, dataset, step_fn, optimizer, scheduler, train_cfg, config_json, checkpoint_dict,
                 eval_dataset, eval_fn, prepare_batch_fn, hooks, resume, auto_resume_path, evacuation) -> None:
        train_config, config_json = _resolve_train_config(train_cfg, config_json)
        self.train_cfg = train_config
        self.settings = _TrainSettings.from_cfg(train_config)
        self._nvtx_open = 0
        self.ema_settings = _EmaSettings.from_cfg(train_config)
        self.step_fn = step_fn
        self.optimizer = optimizer
        self.scheduler = scheduler
        self.dataset = dataset
        self.eval_dataset = eval_dataset
        self.eval_fn = eval_fn
        self.prepare_batch_fn = prepare_batch_fn
        self.hooks = hooks
        if self.settings.checkpoint_async and hooks and hooks.get("on_checkpoint_all_ranks"):
            raise ValueError("All-rank checkpoint hooks require synchronous publication")
        self.checkpoint_dict = checkpoint_dict
        self.resume_mode = str(resume if resume is not None else config_lib.get(train_config, "resume", "none")).lower()
        if self.resume_mode not in {"none", "auto"}:
            raise ValueError("resume must be 'none' or 'auto'")
        if auto_resume_path is not None and self.resume_mode != "auto":
            raise ValueError("auto_resume_path requires resume='auto'")
        if auto_resume_path is not None and checkpoint_dict is None:
            raise ValueError("auto_resume_path requires a preloaded checkpoint")
        self.auto_resume_path = auto_resume_path
        if evacuation is None:
            self.evacuation = EvacuationController(bool(config_lib.get(train_config, "evacuation_enabled", False)),
                                                   signal_name=config_lib.get(train_config, "evacuation_signal", "USR1"))
        elif isinstance(evacuation, bool):
            self.evacuation = EvacuationController(evacuation)
        else:
            self.evacuation = evacuation
        self.evacuation_requested = False
        self.oom_recovery = oom_lib.OomRecoverySettings.from_cfg(train_config)
        self._oom_errors: tuple = (oom_lib.OutOfMemoryError,) if self.oom_recovery.enabled else ()
        self.oom_skipped_steps: set[int] = set()
        self._micro_position: tuple = (0, "fetch")
        self.collector = WarmFreeze()
        self._gather_checkpoint_rng = False

        self.device = ensure_process_device(get_device(train_config))
        model.to(self.device)
        self.model: nn.Module = model
        self.rank = dist_lib.rank()
        self.world_size = dist_lib.world_size()
        self.is_rank0 = dist_lib.rank0()
        self.checkpoint_store = checkpoint_lib.checkpoint_store(self.settings.checkpoint_dir)
        self.checkpoint_publisher = (checkpoint_lib.BackgroundPublisher(self.checkpoint_store,
                                                                        keep_last_k=self.settings.keep_last_k)
                                     if self.settings.checkpoint_async and self.is_rank0 else None)
        self.scaler = make_scaler(self.settings.amp_mode)
        self.cfg_json = config_lib.as_dict(config_json if config_json is not None else train_config)
        self.ctx: Dict[str, Any] = {
            "device": self.device, "rank": self.rank, "world_size": self.world_size,
            "autocast": self._autocast_factory, "scaler": self.scaler, "config": self.cfg_json,
            "config_json": self.cfg_json, "train_cfg": train_config, "model": self.model,
            "evacuation_requested": False, "resume_mode": self.resume_mode, "auto_resume_selected": False,
        }
        self.ema: Optional[EMA] = None
        self.ema_dual: list[EMA] = []
        self._ema_fused_this_step = False
        self.final_ckpt: Optional[Dict[str, Any]] = checkpoint_dict
        self.gpu_health = BackgroundGpuHealth(device=self.device, out_dir=self.settings.out_dir, rank=self.rank,
                                              world_size=self.world_size)
        self._events: Optional[tuple] = None

    # ------------------------------------------------------------------ helpers
    def _autocast_factory(self):
        return autocast_context(self.settings.amp_mode, self.device)

    def _step_ctx(self, step: int) -> Dict[str, Any]:
        return {**self.ctx, "step": step, "optimizer": self.optimizer, "ema": self.ema}

    def _module_for_state(self) -> nn.Module:
        return getattr(self.model, "module", self.model)

    def _on_cuda(self) -> bool:
        return getattr(self.device, "type", "cpu") == "cuda"

    # ------------------------------------------------------------------ setup stages
    def _shard_datasets(self) -> None:
        s = self.settings
        mode = _shard_mode(s.shard_dataset_enabled, s.shard_dataset_mode, "shard_dataset")
        eval_mode = _shard_mode(s.shard_eval_dataset_enabled, s.shard_eval_dataset_mode, "shard_eval_dataset")
        if s.ddp_enabled and mode is not None:
            self.dataset = shard_dataset(self.dataset, rank=self.rank, world_size=self.world_size, mode=mode)
        if s.ddp_enabled and self.eval_dataset is not None and eval_mode is not None:
            self.eval_dataset = shard_dataset(self.eval_dataset, rank=self.rank, world_size=self.world_size,
                                              mode=eval_mode)
        if s.ddp_enabled and s.warn_unsharded and self.is_rank0:
            warn_if_unsharded(self.dataset, enabled=True, name="train dataset")
            warn_if_unsharded(self.eval_dataset, enabled=True, name="eval dataset")

    @staticmethod
    def _parse_compile_cfg(compile_cfg: Any) -> tuple:
        kwargs: Dict[str, Any] = {}
        enabled, preset = True, None
        if isinstance(compile_cfg, Mapping):
            enabled = bool(compile_cfg.get("enabled", True))
            preset = compile_cfg.get("preset", None)
            kwargs = {k: v for k, v in compile_cfg.items() if k not in ("enabled", "preset")}
        elif isinstance(compile_cfg, str):
            preset = compile_cfg
        elif isinstance(compile_cfg, bool):
            enabled = compile_cfg
        return enabled, (str(preset) if preset is not None else None), kwargs

    def _apply_compile(self) -> None:
        """Optional ``torch.compile`` of the model, before data-parallel wrapping (opt-in only)."""

        compile_cfg = config_lib.get(self.train_cfg, "compile", None)
        if not compile_cfg:
            return
        enabled, preset, kwargs = self._parse_compile_cfg(compile_cfg)
        if not enabled:
            return
        if preset is not None:
            kwargs.setdefault("mode", "max-autotune" if preset.lower() in _FULL else preset)
        wraps_only = preset is not None and preset.lower() in _WRAPS_ONLY
        disabled, unwrapped = [], []
        if wraps_only:
            disabled = self._disable_non_wrapped_forwards()
        prev = flags_lib.get_compile_wrap_enabled()
        if not wraps_only:
            flags_lib.set_compile_wrap_enabled(False)
            unwrapped = self._unwrap_compile_wrap_methods()
        try:
            prepare_compile_backend()
            self.model = torch.compile(self.model, **kwargs)
            self.ctx["model"] = self.model
        except Exception as exc:
            for mod, fwd in disabled:
                mod.forward = fwd
            for cls, desc in unwrapped:
                setattr(cls, "forward", desc)
            flags_lib.set_compile_wrap_enabled(prev)
            if self.is_rank0:
                warnings.warn(f"torch.compile failed; falling back to eager: {exc}", RuntimeWarning)

    def _disable_non_wrapped_forwards(self) -> list:
        out = []

        def visit(mod: nn.Module, inside: bool) -> None:
            now = inside or isinstance(getattr(type(mod), "forward", None), flags_lib.compile_wrap)
            if mod is not self.model and not now:
                fwd = mod.forward
                mod.forward = torch._dynamo.disable(mod.forward)
                out.append((mod, fwd))
            for child in mod.children():
                visit(child, now)

        visit(self.model, False)
        return out

    def _unwrap_compile_wrap_methods(self) -> list:
        changed, seen = [], set()
        for mod in self.model.modules():
            cls = type(mod)
            if cls in seen:
                continue
            seen.add(cls)
            desc = getattr(cls, "forward", None)
            if isinstance(desc, flags_lib.compile_wrap):
                setattr(cls, "forward", desc.function)
                changed.append((cls, desc))
        return changed

    def _wrap_ddp(self) -> None:
        if not (self.settings.ddp_enabled and self.world_size > 1):
            return
        assert dist_lib.is_initialized()
        s = self.settings
        if self._on_cuda() and str(torch.distributed.get_backend()).lower() == "nccl":
            from .parallel.ddp import DataParallel

            caps = ([float(s.ddp_bucket_cap_mb)] if s.ddp_bucket_cap_mb is not None else
                    [float(c) for c in s.ddp_bucket_cap_mb_list] if s.ddp_bucket_cap_mb_list else [25.0])
            owners, shard_rest = {}, False
            commit = getattr(self.optimizer, "kb_commit_gradient_plan", None)
            if str(s.comm_transport).lower() in ("fused", "p2p") and callable(commit):
                owners, shard_rest = commit(self.world_size)
            self.model = DataParallel(self.model, bucket_cap_mb=caps, broadcast_buffers=s.ddp_broadcast_buffers,
                                      transport=s.comm_transport, find_unused_parameters=s.find_unused_parameters,
                                      owners=owners, shard_rest=shard_rest)
            if isinstance(self.scaler, FusedGradScaler) and self.model.transport == "fused":
                scaler = self.scaler
                self.model.grad_scale_fn = lambda: scaler._scale
        else:
            from torch.nn.parallel import DistributedDataParallel

            kw: Dict[str, Any] = {"find_unused_parameters": s.find_unused_parameters,
                                  "static_graph": s.ddp_static_graph,
                                  "gradient_as_bucket_view": s.ddp_gradient_as_bucket_view,
                                  "broadcast_buffers": s.ddp_broadcast_buffers}
            if s.ddp_bucket_cap_mb is not None:
                kw["bucket_cap_mb"] = s.ddp_bucket_cap_mb
            if s.ddp_bucket_cap_mb_list is not None:
                kw["bucket_cap_mb_list"] = list(s.ddp_bucket_cap_mb_list)
            if self._on_cuda():
                kw["device_ids"] = [torch.cuda.current_device()]
            self.model = DistributedDataParallel(self.model, **kw)
        self.ctx["model"] = self.model

    # ------------------------------------------------------------------ resume
    def _resume_from_checkpoint(self) -> int:
        ckpt = self.checkpoint_dict
        if not (ckpt and isinstance(ckpt, dict)):
            return 0
        sd = ckpt.get("model")
        if sd is not None:
            self.model.load_state_dict(checkpoint_lib.match_state_dict_to_model(self.model, sd), strict=True)
        for key, target, label in (("optimizer", self.optimizer, "optimizer"),
                                   ("scheduler", self.scheduler, "scheduler")):
            state = ckpt.get(key)
            if target is not None and state is not None:
                try:
                    target.load_state_dict(state)
                except (ValueError, RuntimeError, KeyError) as exc:
                    warnings.warn(f"Failed to restore {label} state from checkpoint: {exc}", RuntimeWarning)
        sc = ckpt.get("scaler")
        if sc is not None and isinstance(self.scaler, GradScaler):
            try:
                self.scaler.load_state_dict(sc)
            except (ValueError, RuntimeError, KeyError) as exc:
                warnings.warn(f"Failed to restore grad-scaler state from checkpoint: {exc}", RuntimeWarning)
        self._restore_ema(ckpt.get("ema"), ckpt.get("ema_dual"))
        rng = ckpt.get("rng")
        if isinstance(rng, Mapping) and "per_rank" in rng:
            states = rng.get("per_rank")
            if isinstance(states, Sequence) and self.rank < len(states):
                rng = states[self.rank]
        if isinstance(rng, Mapping):
            try:
                set_rng_state(dict(rng))
            except (RuntimeError, TypeError, ValueError, KeyError) as exc:
                warnings.warn(f"Failed to restore RNG state from checkpoint: {exc}", RuntimeWarning)
        try:
            if "next_step" in ckpt:
                return int(ckpt["next_step"])
            saved = int(ckpt.get("step", 0))
            conf = ckpt.get("config", {})
            max_steps = int(conf.get("train", conf).get("max_steps", -1))
            # Old terminal checkpoints stored the completed count; periodic ones the last index.
            return saved if saved == max_steps else saved + 1
        except (AttributeError, TypeError, ValueError):
            return 0

    def _load_auto_resume(self) -> Optional[str]:
        if self.resume_mode != "auto":
            return None
        if self.checkpoint_dict is not None:
            if self.auto_resume_path is not None:
                self.ctx["auto_resume_selected"] = True
                return self.auto_resume_path
            return None
        sel = checkpoint_lib.resolve_auto_resume(self.checkpoint_store)
        if sel is None:
            return None
        path, self.checkpoint_dict = sel
        self.ctx["auto_resume_selected"] = True
        return path

    def _restore_one_ema(self, state: Mapping[str, Any], *, fallback_profile: str, fallback_gamma) -> EMA:
        ref = self._module_for_state()
        s = self.ema_settings
        decay = float(state.get("decay", s.target_decay or 0.999))
        prof = str(state.get("profile", fallback_profile)).lower()
        gamma = state.get("gamma", fallback_gamma)
        ema = EMA(ref, decay=decay, profile=prof, gamma=gamma, update_every=s.update_every,
                  offload_to_cpu=s.offload_to_cpu, pin_memory=s.pin_memory,
                  compensate_update_every=s.compensate_update_every)
        shadow = state.get("shadow", {})
        try:
            mapped = checkpoint_lib.match_state_dict_to_model(ref, shadow)
        except (TypeError, AttributeError):
            mapped = shadow
        ema.load_state_dict({
            "decay": decay, "profile": prof, "gamma": gamma, "shadow": mapped,
            "num_updates": state.get("num_updates", 0),
            "step_counter": state.get("step_counter", state.get("num_updates", 0)),
            "update_every": state.get("update_every", s.update_every),
            "compensate_update_every": state.get("compensate_update_every", s.compensate_update_every),
        })
        return ema

    def _restore_ema(self, ema_ckpt, dual_ckpt=None) -> None:
        ref = self._module_for_state()
        s = self.ema_settings
        if ema_ckpt is not None:
            try:
                self.ema = self._restore_one_ema(ema_ckpt, fallback_profile=s.profile, fallback_gamma=s.gamma)
            except (TypeError, ValueError, RuntimeError) as exc:
                warnings.warn(f"Failed to restore EMA from checkpoint: {exc}", RuntimeWarning)
                self.ema = None
        elif s.enabled:
            self.ema = s.build(ref)
        self.ema_dual = []
        if isinstance(dual_ckpt, Sequence) and not isinstance(dual_ckpt, (str, bytes)):
            for i, st in enumerate(dual_ckpt):
                if not isinstance(st, Mapping):
                    continue
                try:
                    self.ema_dual.append(self._restore_one_ema(
                        st, fallback_profile="power", fallback_gamma=s.dual.gamma1 if i == 0 else s.dual.gamma2))
                except (TypeError, ValueError, RuntimeError) as exc:
                    warnings.warn(f"Failed to restore dual EMA #{i} from checkpoint: {exc}", RuntimeWarning)
        elif s.dual.enabled:
            self.ema_dual = s.build_dual(ref)

    # ------------------------------------------------------------------ checkpoints
    def _optimizer_state(self) -> Dict[str, Any]:
        gather = getattr(self.optimizer, "gathered_state_dict", None)
        return gather() if callable(gather) else self.optimizer.state_dict()

    def _build_checkpoint(self, step: int, *, next_step: Optional[int] = None,
                          metrics: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
        module = self._module_for_state()
        try:
            rng: Any = get_rng_state()
            if (self._gather_checkpoint_rng and torch.distributed.is_available() and torch.distributed.is_initialized()
                    and self.world_size > 1):
                gathered: list = [None] * self.world_size
                torch.distributed.all_gather_object(gathered, rng)
                rng = {"per_rank": gathered}
        except RuntimeError:
            if self._gather_checkpoint_rng:
                raise
            rng = None
        ckpt: Dict[str, Any] = {
            "step": step,
            "next_step": step + 1 if next_step is None else int(next_step),
            "model": module.state_dict(),
            "optimizer": self._optimizer_state(),
            "scheduler": self.scheduler.state_dict() if self.scheduler is not None else None,
            "scaler": self.scaler.state_dict() if isinstance(self.scaler, GradScaler) else None,
            "config": self.cfg_json,
            "rng": rng,
            "wall_time": time.time(),
            "metrics": dict(metrics or {}),
        }
        if self.ema is not None:
            ckpt["ema"] = self.ema.state_dict()
        if self.ema_dual:
            ckpt["ema_dual"] = [e.state_dict() for e in self.ema_dual]
        skipped = sorted(s for s in self.oom_skipped_steps if s < ckpt["next_step"])
        if skipped:
            ckpt["oom_skipped_steps"] = skipped
        return ckpt

    def _save_checkpoint(self, step: int, *, next_step: Optional[int] = None, metrics=None, emit_hook: bool = True,
                         background: bool = False) -> tuple:
        ckpt = self._build_checkpoint(step, next_step=next_step, metrics=metrics)
        os.makedirs(self.settings.out_dir, exist_ok=True)
        name = f"step{step:09d}.pt"
        data = checkpoint_lib.serialize(ckpt)
        self._drain_checkpoint()
        if background and self.checkpoint_publisher is not None:
            return self.checkpoint_publisher.submit(name, data, (ckpt, step, emit_hook)), ckpt
        path = checkpoint_lib.publish(self.checkpoint_store, name, data, keep_last_k=self.settings.keep_last_k)
        if emit_hook:
            _emit(self.hooks, "on_checkpoint", path, ckpt, self._step_ctx(step))
        return path, ckpt

    def _announce(self, finished) -> None:
        if finished is None:
            return
        path, (ckpt, step, emit_hook) = finished
        if emit_hook:
            _emit(self.hooks, "on_checkpoint", path, ckpt, self._step_ctx(step))

    def _checkpoint_all_ranks(self, path: str, ckpt: Dict[str, Any], step: int) -> None:
        if not self.hooks or not self.hooks.get("on_checkpoint_all_ranks"):
            return
        dist_lib.barrier()
        _emit(self.hooks, "on_checkpoint_all_ranks", path, ckpt, self._step_ctx(step), suppress_exceptions=False)
        dist_lib.barrier()

    def _poll_checkpoint(self) -> None:
        if self.checkpoint_publisher is not None:
            self._announce(self.checkpoint_publisher.poll())

    def _drain_checkpoint(self) -> None:
        if self.checkpoint_publisher is not None:
            self._announce(self.checkpoint_publisher.wait())

    # ------------------------------------------------------------------ inner loop
    def _make_iterator(self) -> Iterator[Any]:
        if self._on_cuda() and self.settings.prefetch_batches > 0:
            return prefetch(iter(self.dataset), self.device, prefetch=self.settings.prefetch_batches,
                            prepare_fn=self.prepare_batch_fn, threaded=self.settings.prefetch_threaded,
                            pipeline=self.settings.prefetch_pipeline)
        return iter(self.dataset)

    def _profile_sync(self) -> None:
        if self.settings.profile_step_timing and self.settings.profile_step_cuda_sync and self._on_cuda():
            torch.cuda.synchronize(self.device)

    def _profile_start(self, phase: Optional[str] = None) -> float:
        self._profile_sync()
        if self.settings.profile_nvtx and phase is not None and self._on_cuda():
            torch.cuda.nvtx.range_push(f"koochak/{phase}")
            self._nvtx_open += 1
        return time.perf_counter()

    def _profile_add(self, totals: Dict[str, float], key: str, start: float) -> float:
        self._profile_sync()
        if self._nvtx_open:
            torch.cuda.nvtx.range_pop()
            self._nvtx_open -= 1
        elapsed = time.perf_counter() - start
        if self.settings.profile_step_timing:
            totals[key] = totals.get(key, 0.0) + elapsed
        return elapsed

    def _run_micro_steps(self, step: int, it: Iterator[Any], *, collect_rank_timing: bool) -> _MicroStats:
        stats = _MicroStats()
        autocast_factory = self.ctx.get("autocast")
        use_prefetch = self._on_cuda() and self.settings.prefetch_batches > 0
        n = self.settings.grad_accum
        for micro in range(n):
            sync_cm = self.model.no_sync() if (hasattr(self.model, "no_sync") and micro < n - 1) else nullcontext()
            ac = autocast_factory() if (callable(autocast_factory) and not self.settings.autocast_in_step_fn) \
                else nullcontext()
            with sync_cm, ac:
                self._micro_position = (micro, "fetch")
                t0 = self._profile_start("batch_wait")
                batch = next(it) if use_prefetch else to_device(next(it), self.device)
                stats.batch_wait_s += self._profile_add(stats.profile_timing_totals, "profile_loop_batch_wait_time_s",
                                                        t0)
                for k, v in _skip_counts(batch).items():
                    stats.skip_count_totals[k] = stats.skip_count_totals.get(k, 0.0) + float(v)
                self._micro_position = (micro, "step_fn")
                t0 = self._profile_start("step_fn")
                out = self.step_fn(self.model, batch, self._step_ctx(step))
                self._profile_add(stats.profile_timing_totals, "profile_loop_step_fn_time_s", t0)
                if collect_rank_timing and isinstance(out, Mapping):
                    for key in self.settings.rank_timing_extra_keys:
                        v = out.get(key)
                        if v is None:
                            continue
                        if isinstance(v, torch.Tensor):
                            v = float(v.detach())
                        stats.extra_timing_totals[key] = stats.extra_timing_totals.get(key, 0.0) + float(v)
                if not isinstance(out, Mapping) or "loss" not in out:
                    raise RuntimeError("step_fn must return a dict containing a 'loss' Tensor")
                if not isinstance(out["loss"], torch.Tensor):
                    raise RuntimeError("step_fn returned a 'loss' that is not a torch.Tensor")
                loss = out["loss"] / n
            self._micro_position = (micro, "backward")
            t0 = self._profile_start("backward")
            self.scaler.scale(loss).backward()
            self._profile_add(stats.profile_timing_totals, "profile_loop_backward_time_s", t0)
            d = loss.detach()
            stats.total_loss = d if stats.total_loss is None else stats.total_loss + d
            if self.settings.scalarize_loss_every_step:
                stats.total_loss_scalar = float(stats.total_loss)
            stats.out = out
        return stats

    def _nonfinite_names(self) -> list:
        bad = []
        for name, p in self.model.named_parameters():
            if p.grad is not None and torch.is_floating_point(p.grad) and not torch.isfinite(p.grad).all():
                bad.append(name)
        return bad

    def _check_nonfinite_grads(self, step: int) -> None:
        every = self.settings.nonfinite_grad_check_every
        if every <= 0 or step % every != 0:
            return
        bad = self._nonfinite_names()
        if bad:
            raise FloatingPointError("Gradient entries contain NaN or infinity; optimizer step stopped: "
                                     + ", ".join(bad))

    def _native_grads(self) -> Optional[list]:
        if not self._on_cuda():
            return None
        grads = []
        for p in self.model.parameters():
            if p.grad is None:
                continue
            g = p.grad
            if not (g.is_cuda and g.dtype == torch.float32 and g.is_contiguous() and g.layout == torch.strided):
                return None
            grads.append(g)
        if not grads:
            return None
        from .ops._ext import available

        return grads if available() else None

    def _gradient_gate(self, step: int, stats: _MicroStats) -> None:
        """Unscale -> optional finite check -> optional clip (reference: koochak/loop.py:1612-1637)."""

        s = self.settings
        clip = s.grad_clip_norm is not None
        grads = self._native_grads()
        fused_opt = bool(getattr(self.optimizer, "kb_fused", False)) or bool(
            getattr(getattr(self.optimizer, "inner", None), "kb_fused", False))

        t0 = self._profile_start("unscale")
        gate_stats = None
        dp = self.model if getattr(self.model, "fused_gate_available", None) is not None else None
        if dp is not None and grads is not None and dp.fused_gate_available():
            # The fused all-reduce already averaged, unscaled and measured the
            # gradients: the gate is one small kernel and one host read.
            gate_stats = dp.fused_gate(s.grad_clip_norm)
            if isinstance(self.scaler, FusedGradScaler):
                self.scaler.mark_unscaled(self.optimizer, gate_stats)
        elif isinstance(self.scaler, FusedGradScaler) and grads is not None:
            self.scaler.unscale_(self.optimizer, max_norm=s.grad_clip_norm)
            gate_stats = self.scaler.last_stats
        elif isinstance(self.scaler, GradScaler):
            self.scaler.unscale_(self.optimizer)
        self._profile_add(stats.profile_timing_totals, "profile_loop_unscale_time_s", t0)

        t0 = self._profile_start("nonfinite_grad_check")
        self._check_nonfinite_grads(step)
        self._profile_add(stats.profile_timing_totals, "profile_loop_nonfinite_grad_check_time_s", t0)

        t0 = self._profile_start("grad_clip")
        if clip:
            if grads is None:
                clipping = clip_grad_norm_(self.model.parameters(), float(s.grad_clip_norm))
            elif gate_stats is not None:
                clipping = self._clip_from_stats(gate_stats, grads, fused_opt)
            else:
                res = fused_grad_gate(grads, max_norm=float(s.grad_clip_norm), check_finite=True)
                clipping = res.stats
                if res.coef_tensor is not None:
                    self._apply_coef(res.coef_tensor, grads, fused_opt)
            if isinstance(clipping, GradientClipStats):
                if stats.out is None:
                    stats.out = {}
                stats.out.update(grad_norm=clipping.norm, grad_clip_coefficient=clipping.coefficient,
                                 grad_clip_scaled_norm=int(clipping.used_scaled_norm))
        self._profile_add(stats.profile_timing_totals, "profile_loop_grad_clip_time_s", t0)

    @staticmethod
    def _raise_if_comm_failed(gate_stats: torch.Tensor) -> None:
        if float(gate_stats[3]) != 0.0:
            from .ops._ext import check_status

            check_status(int(gate_stats.device.index or 0))
            raise RuntimeError(f"gradient all-reduce reported device status {int(float(gate_stats[3]))}")

    def _apply_coef(self, coef: torch.Tensor, grads: list, fused_opt: bool) -> None:
        if fused_opt:
            self.optimizer.kb_grad_scale = coef
        else:
            torch._foreach_mul_(grads, coef)

    def _clip_from_stats(self, out: torch.Tensor, grads: list, fused_opt: bool) -> GradientClipStats:
        vals = out.tolist()
        norm, coef, bad = (float(v) for v in vals[:3])
        if len(vals) > 3 and vals[3] != 0.0:
            self._raise_if_comm_failed(out)
        if bad or not math.isfinite(norm) or 0.0 < coef < torch.finfo(torch.float32).tiny:
            # fp16 overflow or huge values: the reference path decides (and raises on inf/nan).
            return clip_grad_norm_(self.model.parameters(), float(self.settings.grad_clip_norm))
        self._apply_coef(out[1:2], grads, fused_opt)
        return GradientClipStats(norm, coef, False)

    def _maybe_fuse_ema(self, step: int) -> None:
        self._ema_fused_this_step = False
        if self.ema is None or self.ema_dual or isinstance(self.scaler, GradScaler):
            return
        opt = self.optimizer
        target = opt if getattr(opt, "kb_fused", False) else getattr(opt, "inner", None)
        if target is None or not getattr(target, "kb_fused", False) or not self.ema.fusable():
            return
        if self.world_size > 1 and getattr(target, "_distributed", False):
            return
        s = self.ema_settings
        decay = None if s.profile == "power" else s.warmed_decay(step)
        target.kb_ema = self.ema.begin_fused_update(self._module_for_state(), decay)
        self._ema_fused_this_step = True

    def _update_ema(self, step: int) -> None:
        s = self.ema_settings
        all_ranks = bool(self.hooks and self.hooks.get("on_checkpoint_all_ranks"))
        if self.ema is None and s.enabled and (self.is_rank0 or all_ranks):
            self.ema = s.build(self._module_for_state())
        if not self.ema_dual and s.dual.enabled and (self.is_rank0 or all_ranks):
            self.ema_dual = s.build_dual(self._module_for_state())
        module = self._module_for_state()
        if self.ema is not None and not self._ema_fused_this_step:
            if s.profile == "power":
                self.ema.update(module)
            else:
                self.ema.update(module, decay=s.warmed_decay(step))
        for e in self.ema_dual:
            e.update(module)
        self._ema_fused_this_step = False

    def _step_scheduler(self) -> None:
        if self.scheduler is None or self.settings.scheduler_step_policy != "step":
            return
        try:
            self.scheduler.step()
        except TypeError:
            pass  # schedulers that need a metric step after eval

    def _emit_rank_timing(self, step: int, stats: _MicroStats, step_time_s: float) -> None:
        payload: Dict[str, Any] = {"rank": self.rank, "batch_wait_s": float(stats.batch_wait_s),
                                   "step_compute_s": float(max(0.0, step_time_s - stats.batch_wait_s)),
                                   "total_step_s": float(step_time_s)}
        for k in self.settings.rank_timing_extra_keys:
            payload[k] = float(stats.extra_timing_totals.get(k, stats.profile_timing_totals.get(k, 0.0)))
        gathered: list = [None] * self.world_size
        torch.distributed.all_gather_object(gathered, payload)
        if self.is_rank0:
            print(_format_rank_timing([g for g in gathered if isinstance(g, dict)], step,
                                      self.settings.rank_timing_extra_keys))

    def _build_logs(self, step: int, stats: _MicroStats, step_time_s: float) -> tuple:
        loss_value: Any = stats.total_loss_scalar
        if loss_value is None:
            loss_value = stats.total_loss if stats.total_loss is not None else 0.0
        minimal: Dict[str, Any] = {"loss": loss_value, "lr": get_lr(self.optimizer), "step_time_s": step_time_s,
                                   "step": step}
        if not (self.is_rank0 and step % self.settings.log_every == 0):
            return None, minimal
        loss_scalar = (float(stats.total_loss) if stats.total_loss_scalar is None and stats.total_loss is not None
                       else float(stats.total_loss_scalar or 0.0))
        stats.total_loss_scalar = loss_scalar
        extra = {}
        for k, v in (stats.out or {}).items():
            if k == "loss":
                continue
            extra[k] = float(v.detach()) if isinstance(v, torch.Tensor) else v
        prof = {k: float(v) for k, v in stats.profile_timing_totals.items() if k.startswith("profile_loop_")}
        full = {"loss": loss_scalar, "lr": get_lr(self.optimizer), "step_time_s": step_time_s,
                **{k: float(v) for k, v in stats.skip_count_totals.items()}, **extra, **prof, "step": step}
        return full, full

    # ------------------------------------------------------------------ health
    def _handle_health_failure(self, step: int, failures: list) -> None:
        self.gpu_health.close()
        completed = step + 1
        bad_nodes = self.gpu_health.bad_nodes_from_failures(failures)
        metrics = {"gpu_health": {"event": "gpu_health_shutdown", "failures": failures, "bad_nodes": bad_nodes,
                                  "slurm_action": self.gpu_health.slurm_action,
                                  "slurm_disabled": self.gpu_health.slurm_disabled}}
        self._gather_checkpoint_rng = True
        try:
            if self.is_rank0:
                path, ckpt = self._save_checkpoint(completed, next_step=completed, metrics=metrics, emit_hook=False)
            else:
                ckpt = self._build_checkpoint(completed, next_step=completed, metrics=metrics)
                path = checkpoint_lib.checkpoint_path(self.checkpoint_store, f"step{completed:09d}.pt")
        finally:
            self._gather_checkpoint_rng = False
        self.final_ckpt = ckpt
        dist_lib.barrier()
        if self.is_rank0:
            _emit(self.hooks, "on_checkpoint", path, ckpt, self._step_ctx(completed))
            summary = self.gpu_health.write_failure_summary(step=completed, failures=failures, checkpoint_path=path)
            print(f"[gpu-health] FAIL step={step} {summarize_failures_for_stdout(failures)}", flush=True)
            print(f"[gpu-health] checkpoint={path} summary={summary} slurm_action={self.gpu_health.slurm_action} "
                  f"bad_nodes={','.join(bad_nodes)}", flush=True)
        dist_lib.barrier()
        if self.is_rank0:
            results = self.gpu_health.perform_slurm_recovery(failures)
            if results:
                print(f"[gpu-health] slurm_results={json.dumps(results, sort_keys=True)}", flush=True)
        elif (os.environ.get("SLURM_JOB_ID") and not self.gpu_health.slurm_disabled
              and self.gpu_health.slurm_action in {"requeue", "cancel"}):
            time.sleep(30.0)  # give rank 0 time to mutate the Slurm job before teardown
        raise SystemExit(self.gpu_health.exit_code)

    def _reconcile_stop_requests(self, step: int) -> None:
        self.gpu_health.update_step(step)
        local = self.gpu_health.failures()
        evacuate, health = self.evacuation.reconcile_requests(bool(local))
        self.evacuation_requested = evacuate
        self.ctx["evacuation_requested"] = evacuate
        if health:
            gathered = [local]
            if dist_lib.is_initialized():
                gathered = [None] * self.world_size
                torch.distributed.all_gather_object(gathered, local)
            self._handle_health_failure(step, [f for rank_failures in gathered for f in rank_failures])

    # ------------------------------------------------------------------ OOM
    def _load_oom_records(self, start_step: int) -> None:
        steps = sorted(oom_lib.recorded_steps(self.checkpoint_store)) if self.is_rank0 else None
        if self.world_size > 1 and dist_lib.is_initialized():
            box = [steps]
            torch.distributed.broadcast_object_list(box, src=0)
            steps = box[0]
        self.oom_skipped_steps = set(steps or ())
        pending = [s for s in sorted(self.oom_skipped_steps) if start_step <= s < self.settings.max_steps]
        if pending and self.is_rank0:
            shown = ", ".join(str(s) for s in pending[:20]) + (", ..." if len(pending) > 20 else "")
            print(f"[oom] {len(pending)} step(s) recorded as OOM-skipped by earlier attempts will be skipped: {shown}",
                  flush=True)

    def _oom_record(self, step: int, exc: BaseException) -> Dict[str, Any]:
        micro, phase = self._micro_position
        decision = oom_lib.decide(self.oom_recovery, self.oom_skipped_steps, step, distributed=self.world_size > 1,
                                  during_fetch=phase == "fetch")
        memory, summary = oom_lib.memory_report(self.device)
        record = {"v": 1, "step": step, "rank": self.rank, "world_size": self.world_size, "phase": phase,
                  "micro_step": micro, "grad_accum": self.settings.grad_accum, "action": decision.action,
                  "reason": decision.reason, "consecutive": decision.consecutive,
                  "max_consecutive": self.oom_recovery.max_consecutive, "skipped_total": decision.skipped_total,
                  "error_type": type(exc).__name__, "message": oom_lib.short_message(exc), "memory": memory,
                  "memory_summary": summary, "wall_time": time.time()}
        print(oom_lib.format_record(record), flush=True)
        return record

    def _recover_from_oom(self, step: int, it: Iterator[Any], record: Dict[str, Any]) -> bool:
        self.optimizer.zero_grad(set_to_none=True)
        oom_lib.release_memory(self.device)
        oom_lib.write_record(self.checkpoint_store, record)  # durable before anything that can fail
        self.oom_skipped_steps.add(step)
        _emit(self.hooks, "on_oom", record, self._step_ctx(step))
        if self.world_size > 1:
            print(f"[oom] rank={self.rank} exiting with code {OOM_RESTART_EXIT_CODE}; resubmit with resume=auto to "
                  "continue from the last checkpoint", flush=True)
            raise SystemExit(OOM_RESTART_EXIT_CODE)
        if record["phase"] != "fetch":
            if not self._drain_micro_batches(it, self.settings.grad_accum - (int(record["micro_step"]) + 1)):
                return False
        self._step_scheduler()
        if record["action"] == oom_lib.RESTART:
            self._checkpoint_and_exit_after_oom(step)
        return self._finish_step(step, {})

    def _replay_oom_skip(self, step: int, it: Iterator[Any]) -> bool:
        if not self._drain_micro_batches(it, self.settings.grad_accum):
            return False
        self._step_scheduler()
        if self.is_rank0:
            print(f"[oom] step={step} skipped: recorded as OOM by an earlier attempt", flush=True)
        return self._finish_step(step, {})

    @staticmethod
    def _drain_micro_batches(it: Iterator[Any], count: int) -> bool:
        for _ in range(count):
            try:
                next(it)
            except StopIteration:
                return False
        return True

    def _checkpoint_and_exit_after_oom(self, step: int) -> None:
        completed = step + 1
        self._gather_checkpoint_rng = True
        try:
            path, self.final_ckpt = self._save_checkpoint(completed, next_step=completed, emit_hook=False)
        finally:
            self._gather_checkpoint_rng = False
        _emit(self.hooks, "on_checkpoint", path, self.final_ckpt, self._step_ctx(completed))
        print(f"[oom] checkpoint={path} next_step={completed}; exiting with code {OOM_RESTART_EXIT_CODE} so a "
              "resubmit starts with a fresh CUDA allocator", flush=True)
        raise SystemExit(OOM_RESTART_EXIT_CODE)

    # ------------------------------------------------------------------ eval
    def _maybe_run_eval(self, step: int) -> None:
        if self.eval_fn is None or self.eval_dataset is None or self.settings.eval_every <= 0:
            return
        at = step + int(self.settings.intervals_use_completed_steps)
        if at == 0 and not self.settings.eval_at_step_zero:
            return
        if at % self.settings.eval_every != 0:
            return
        if self.ema is not None and self.ema_settings.eval_with_ema:
            metrics = self._eval_with_ema(step)
        else:
            metrics = self.eval_fn(self.model, self.eval_dataset, self._step_ctx(step))
        if self.scheduler is not None and self.settings.scheduler_step_policy == "eval":
            self.scheduler.step(metrics.get("val_loss", None))
        if self.is_rank0:
            _emit(self.hooks, "on_eval_end", metrics, self._step_ctx(step))

    def _eval_with_ema(self, step: int) -> Dict[str, float]:
        assert self.ema is not None and self.eval_fn is not None
        module = self._module_for_state()
        try:
            self.ema.store(module)
            self.ema.copy_to(module)
            return self.eval_fn(self.model, self.eval_dataset, self._step_ctx(step))
        finally:
            self.ema.restore(module)

    # ------------------------------------------------------------------ orchestration
    def run(self) -> Dict[str, Any]:
        it: Optional[Iterator[Any]] = None
        try:
            self.evacuation.install()
            if self.evacuation.already_evacuated:
                print("[evacuation] run already evacuated; exiting before training", flush=True)
                raise SystemExit(EVACUATION_EXIT_CODE)
            self.gpu_health.start()
            self._shard_datasets()
            resume_path = self._load_auto_resume()
            _emit(self.hooks, "on_train_start", self.ctx, suppress_exceptions=False)
            self._apply_compile()
            self._wrap_ddp()
            if self.is_rank0:
                c = _parameter_counts(self.model)
                print(f"[training] Model parameters — total: {c['total']:,} | trainable: {c['trainable']:,} | "
                      f"frozen: {c['frozen']:,}")
            start = self._resume_from_checkpoint()
            if self.oom_recovery.enabled:
                self._load_oom_records(start)
            if resume_path is not None and self.is_rank0:
                _emit(self.hooks, "on_resume_checkpoint", resume_path, self.checkpoint_dict, self._step_ctx(start))
            next_step = start
            it = self._make_iterator()
            interrupted = False
            for step in range(start, self.settings.max_steps):
                if not self._run_step(step, it):
                    break
                next_step = step + 1
                if self.evacuation_requested:
                    interrupted = True
                    break
            self.gpu_health.close()
            self._reconcile_stop_requests(next_step - 1)
            interrupted = interrupted or self.evacuation_requested
            # Terminal checkpoint: a completed-update cursor (step == next_step).
            self._gather_checkpoint_rng = True
            terminal = checkpoint_lib.checkpoint_path(self.checkpoint_store, f"step{next_step:09d}.pt")
            if self.is_rank0:
                terminal, self.final_ckpt = self._save_checkpoint(next_step, next_step=next_step, emit_hook=False)
            else:
                self.final_ckpt = self._build_checkpoint(next_step, next_step=next_step)
            self._gather_checkpoint_rng = False
            if torch.distributed.is_available() and torch.distributed.is_initialized():
                dist_lib.barrier()
            if self.is_rank0:
                _emit(self.hooks, "on_checkpoint", terminal, self.final_ckpt, self._step_ctx(next_step))
            self._checkpoint_all_ranks(terminal, self.final_ckpt, next_step)
            if interrupted:
                if self.is_rank0:
                    _emit(self.hooks, "on_evacuation", terminal, self.final_ckpt, self._step_ctx(next_step))
                _emit(self.hooks, "on_train_end", self.ctx)
                if torch.distributed.is_available() and torch.distributed.is_initialized():
                    dist_lib.barrier()
                self.evacuation.mark_evacuated()
                raise SystemExit(EVACUATION_EXIT_CODE)
            _emit(self.hooks, "on_train_end", self.ctx)
        except Exception as exc:
            _emit(self.hooks, "on_exception", exc, self.ctx)
            raise
        finally:
            close_it = getattr(it, "close", None) if it is not None else None
            with ExitStack() as cleanup:
                if callable(close_it):
                    cleanup.callback(close_it)
                if self.checkpoint_publisher is not None:
                    cleanup.callback(self.checkpoint_publisher.close)
                cleanup.callback(self.evacuation.uninstall)
                cleanup.callback(self.gpu_health.close)
        assert self.final_ckpt is not None
        return self.final_ckpt

    def _device_timer_start(self) -> None:
        if self.settings.device_timing and self._on_cuda():
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            self._events = (start, end)

    def _device_timer_stop(self) -> Optional[float]:
        if self._events is None:
            return None
        start, end = self._events
        end.record()
        end.synchronize()
        self._events = None
        return float(start.elapsed_time(end))

    def _run_step(self, step: int, it: Iterator[Any]) -> bool:
        if step in self.oom_skipped_steps:
            return self._replay_oom_skip(step, it)
        step_start = self._profile_start()
        self._device_timer_start()
        totals: Dict[str, float] = {}
        t0 = self._profile_start("setup_zero_grad")
        self.model.train()
        self.optimizer.zero_grad(set_to_none=True)
        self._profile_add(totals, "profile_loop_setup_zero_grad_time_s", t0)
        collect = (self.settings.ddp_enabled and self.world_size > 1 and self.settings.rank_timing_every > 0
                   and step % self.settings.rank_timing_every == 0)
        oom = None
        try:
            stats = self._run_micro_steps(step, it, collect_rank_timing=collect)
        except StopIteration:
            return False
        except self._oom_errors as exc:
            oom = self._oom_record(step, exc)
            if oom["action"] == oom_lib.FAIL:
                raise
        if oom is not None:
            return self._recover_from_oom(step, it, oom)
        for k, v in totals.items():
            stats.profile_timing_totals[k] = stats.profile_timing_totals.get(k, 0.0) + v

        self._gradient_gate(step, stats)

        t0 = self._profile_start("ema_wait")
        if self.ema is not None:
            self.ema.wait_before_param_mutation()
        for e in self.ema_dual:
            e.wait_before_param_mutation()
        self._profile_add(stats.profile_timing_totals, "profile_loop_ema_wait_time_s", t0)

        self._maybe_fuse_ema(step)
        t0 = self._profile_start("optimizer_step")
        self.scaler.step(self.optimizer)
        self._profile_add(stats.profile_timing_totals, "profile_loop_optimizer_step_time_s", t0)
        t0 = self._profile_start("scaler_update")
        self.scaler.update()
        self._profile_add(stats.profile_timing_totals, "profile_loop_scaler_update_time_s", t0)
        t0 = self._profile_start("ema_update")
        self._update_ema(step)
        self._profile_add(stats.profile_timing_totals, "profile_loop_ema_update_time_s", t0)
        t0 = self._profile_start("scheduler")
        self._step_scheduler()
        self._profile_add(stats.profile_timing_totals, "profile_loop_scheduler_time_s", t0)

        self._profile_sync()
        step_time_s = time.perf_counter() - step_start
        device_ms = self._device_timer_stop()
        if collect:
            self._emit_rank_timing(step, stats, step_time_s)
        t0 = self._profile_start("log_build")
        full, minimal = self._build_logs(step, stats, step_time_s)
        if device_ms is not None:
            minimal["step_device_ms"] = device_ms
            if full is not None:
                full["step_device_ms"] = device_ms
        built = self._profile_add(stats.profile_timing_totals, "profile_loop_log_build_time_s", t0)
        if self.settings.profile_step_timing:
            if full is not None:
                full["profile_loop_log_build_time_s"] = built
            minimal["profile_loop_log_build_time_s"] = built
        t0 = self._profile_start("log_emit")
        _emit(self.hooks, "on_update_end", minimal, self._step_ctx(step))
        if full is not None:
            _emit(self.hooks, "on_log", full, self._step_ctx(step))
        _emit(self.hooks, "on_step_end", minimal, self._step_ctx(step))
        self._profile_add(stats.profile_timing_totals, "profile_loop_log_emit_time_s", t0)
        self.collector.update()
        return self._finish_step(step, stats.profile_timing_totals)

    def _finish_step(self, step: int, totals: Dict[str, float]) -> bool:
        t0 = self._profile_start("health_check")
        self._reconcile_stop_requests(step)
        self._profile_add(totals, "profile_loop_health_check_time_s", t0)
        t0 = self._profile_start("eval")
        self._maybe_run_eval(step)
        self._profile_add(totals, "profile_loop_eval_time_s", t0)
        if self.evacuation_requested:
            return True
        t0 = self._profile_start("checkpoint")
        at = step + int(self.settings.intervals_use_completed_steps)
        terminal_due = self.settings.intervals_use_completed_steps and at == self.settings.max_steps
        if at > 0 and at % self.settings.ckpt_every == 0 and not terminal_due:
            self._gather_checkpoint_rng = True
            try:
                if self.is_rank0:
                    path, ckpt = self._save_checkpoint(at, next_step=step + 1,
                                                       background=self.settings.checkpoint_async)
                    self.final_ckpt = ckpt
                else:
                    ckpt = self._build_checkpoint(at, next_step=step + 1)
                    path = checkpoint_lib.checkpoint_path(self.checkpoint_store, f"step{at:09d}.pt")
            finally:
                self._gather_checkpoint_rng = False
            if not self.settings.checkpoint_async:
                dist_lib.barrier()  # keep peers out of the next step until rank 0 has published
            self._checkpoint_all_ranks(path, ckpt, at)
        self._poll_checkpoint()
        self._profile_add(totals, "profile_loop_checkpoint_time_s", t0)
        return True
