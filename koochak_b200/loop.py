"""``training_loop``: the function-first training runtime.

(public contract of reference koochak/loop.py:437-476: the same keyword
signature, hook names and payloads, config keys, checkpoint format, exit
codes)

The caller supplies a model, a dataset, ``step_fn(model, batch, ctx) ->
{"loss": tensor, ...}``, an optimizer and the ``train`` config. The run is
assembled from parts, most of them in ``koochak_b200.runtime``:

* ``LoopSettings`` / ``EmaSettings`` -- the ``train.*`` keys, read once;
* ``_Profiler`` -- optional per-phase wall time (and NVTX ranges), reported
  as ``profile_loop_*_time_s``;
* ``_MicroSteps`` -- gradient accumulation: ``no_sync`` on all but the last
  micro-batch, autocast, ``step_fn``, scaled backward (on the native
  data-parallel path backward launches the bucket reductions from gradient
  hooks);
* ``GradientGate`` -- unscale, finite check and clip, from the fused
  reduction's statistics when there are any (one 16-byte read per step);
* the update -- EMA snapshot wait, optimizer (the fused optimizers take the
  clip coefficient and the GPU EMA into their own kernels), scaler, EMA,
  scheduler;
* ``CheckpointKeeper`` -- every rank collects (optimizer state gathered from
  its owners), rank 0 publishes ``stepNNNNNNNNN.pt`` + ``.ready.json``;
* ``_StopControl`` -- after every update, one small cross-rank reduction
  agrees on evacuation (SIGUSR1 / the runner's request file) and GPU-health
  failures; an agreed stop checkpoints and exits 75 or 42;
* ``_OomGuard`` -- opt-in recovery from CUDA out-of-memory inside a step.
"""

from __future__ import annotations

import json
import os
import statistics
import time
import warnings
from contextlib import ExitStack, nullcontext
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterable, Iterator, List, Mapping, Optional, Sequence, Tuple

import torch
import torch.nn as nn
from torch.amp import GradScaler
from torch.optim import Optimizer
from torch.optim.lr_scheduler import _LRScheduler

from . import oom as oom_lib
from .core import dist as dist_lib
from .core import hooks as hooks_lib
from .core.precision import FusedGradScaler, Scaler as make_scaler, autocast_context, prepare_compile_backend
from .data.iterable import prefetch, to_device
from .data.sharding import shard_dataset, warn_if_unsharded
from .health.background import BackgroundGpuHealth
from .health.gpu import summarize_failures_for_stdout
from .interruption import EVACUATION_EXIT_CODE, OOM_RESTART_EXIT_CODE, EvacuationController
from .runtime.checkpoints import CheckpointKeeper, EmaBuilder, restore_ema, restore_training_state
from .runtime.gate import GradientGate
from .runtime.graphed_step import GraphedStep
from .runtime.settings import EmaSettings, LoopSettings, shard_mode
from .storage import checkpoint as checkpoint_lib
from .utils import config as config_lib
from .utils import flags as flags_lib
from .utils.collector import WarmFreeze
from .utils.device import ensure_process_device, get_device, get_lr
from .utils.ema import EMA

__all__ = ["training_loop", "StepFn", "EvalFn", "BatchPrepareFn"]

StepFn = Callable[[nn.Module, Any, Mapping[str, Any]], Dict[str, Any]]
EvalFn = Callable[[nn.Module, Iterable, Mapping[str, Any]], Dict[str, float]]
BatchPrepareFn = Callable[[Any], Any]

_ROOT_SECTIONS = ("data", "optim", "logging", "wandb", "entry")
_COMPILE_WRAPS_ONLY = frozenset({"wraps", "wraps-only", "merge-wraps", "merge_wraps"})
_COMPILE_FULL = frozenset({"full", "full-model", "full_model"})
_RANK_TIMING = ("batch_wait_s", "step_compute_s", "total_step_s")


def training_loop(*, model: nn.Module, dataset: Iterable, step_fn: StepFn, optimizer: Optimizer,
                  scheduler: Optional[_LRScheduler] = None, train_cfg: Mapping[str, Any] | Any,
                  config_json: Optional[Mapping[str, Any]] = None, checkpoint_dict: Optional[Dict[str, Any]] = None,
                  eval_dataset: Optional[Iterable] = None, eval_fn: Optional[EvalFn] = None,
                  prepare_batch_fn: Optional[BatchPrepareFn] = None,
                  hooks: Optional[Dict[str, list[Callable]]] = None, resume: Optional[str] = None,
                  auto_resume_path: Optional[str] = None,
                  evacuation: Optional[EvacuationController | bool] = None) -> Dict[str, Any]:
    """Train until ``train.max_steps`` or dataset exhaustion; return the final checkpoint dict."""

    return _Run(model=model, dataset=dataset, step_fn=step_fn, optimizer=optimizer, scheduler=scheduler,
                train_cfg=train_cfg, config_json=config_json, checkpoint_dict=checkpoint_dict,
                eval_dataset=eval_dataset, eval_fn=eval_fn, prepare_batch_fn=prepare_batch_fn, hooks=hooks,
                resume=resume, auto_resume_path=auto_resume_path, evacuation=evacuation).execute()


# ----------------------------------------------------------------------------- small helpers


def _split_root_config(train_cfg: Any, config_json: Optional[Mapping[str, Any]]):
    """A whole root config passed as ``train_cfg`` is still accepted (deprecated): use its ``train`` part."""

    is_root = (("train" in train_cfg and any(k in train_cfg for k in _ROOT_SECTIONS)) if isinstance(train_cfg, Mapping)
               else all(hasattr(train_cfg, k) for k in ("train",) + _ROOT_SECTIONS))
    if is_root:
        warnings.warn("training_loop now expects train_cfg only; passing the full root config is deprecated.",
                      DeprecationWarning)
        return config_lib.get(train_cfg, "train", {}) or {}, config_json or train_cfg
    return train_cfg or {}, config_json


def _sum_of(value: Any) -> float:
    if isinstance(value, torch.Tensor):
        return float(value.detach().to(torch.float32).sum().item())
    if isinstance(value, (list, tuple)):
        return float(sum(float(x) for x in value))
    return float(value)


def _checked(out: Any) -> Mapping[str, Any]:
    if not isinstance(out, Mapping) or "loss" not in out:
        raise RuntimeError("step_fn must return a dict containing a 'loss' Tensor")
    if not isinstance(out["loss"], torch.Tensor):
        raise RuntimeError("step_fn returned a 'loss' that is not a torch.Tensor")
    return out


def _skip_counters(batch: Any) -> Dict[str, float]:
    """``*_skip_count`` entries a dataset put into a dict batch, summed."""

    if not isinstance(batch, Mapping):
        return {}
    return {str(k): _sum_of(v) for k, v in batch.items() if str(k).endswith("_skip_count")}


def _rank_timing_line(entries: List[Dict[str, Any]], step: int, keys: Sequence[str]) -> str:
    def part(key: str) -> str:
        if not entries:
            return f"{key}=n/a"
        ranked = sorted((float(e.get(key, 0.0)), int(e.get("rank", 0))) for e in entries)
        fastest, (slowest, who) = ranked[0][0], ranked[-1]
        middle = statistics.median(v for v, _ in ranked)
        return f"{key}={fastest:.3f}/{middle:.3f}/{slowest:.3f}@r{who} span={slowest - fastest:.3f}"

    return f"[rank-timing] step={step} " + " ".join(part(k) for k in (*_RANK_TIMING, *keys))


def _parameter_counts(module: nn.Module) -> Tuple[int, int]:
    inner = getattr(module, "module", module)
    total = sum(p.numel() for p in inner.parameters())
    return total, sum(p.numel() for p in inner.parameters() if p.requires_grad)


class _Profiler:
    """Per-phase wall time (``profile_step_fn_timing``) with optional CUDA sync and NVTX ranges."""

    def __init__(self, settings: LoopSettings, on_cuda: bool, device: torch.device) -> None:
        self.timing = settings.profile_step_timing
        self.sync = settings.profile_step_timing and settings.profile_step_cuda_sync and on_cuda
        self.nvtx = settings.profile_nvtx and on_cuda
        # Named host ranges for torch.profiler (the reference's KAVEH_PROFILE_RANGES switch).
        self.ranges = os.environ.get("KAVEH_PROFILE_RANGES", "").lower() in {"1", "true", "yes", "on"}
        self._ranges: List[Any] = []
        self.device = device
        self._open = 0

    def barrier(self) -> None:
        if self.sync:
            torch.cuda.synchronize(self.device)

    def start(self, phase: Optional[str] = None) -> float:
        self.barrier()
        if self.nvtx and phase is not None:
            torch.cuda.nvtx.range_push(f"koochak/{phase}")
            self._open += 1
        if self.ranges and phase is not None:  # every stop() pairs with a start() that named its phase
            rf = torch.autograd.profiler.record_function(f"loop.{phase}")
            rf.__enter__()
            self._ranges.append(rf)
        return time.perf_counter()

    def stop(self, totals: Dict[str, float], key: str, began: float) -> float:
        self.barrier()
        if self._open:
            torch.cuda.nvtx.range_pop()
            self._open -= 1
        if self._ranges:
            self._ranges.pop().__exit__(None, None, None)
        took = time.perf_counter() - began
        if self.timing:
            totals[key] = totals.get(key, 0.0) + took
        return took

    def run(self, totals: Dict[str, float], key: str, thunk: Callable[[], Any]) -> Any:
        began = self.start(key[len("profile_loop_"):-len("_time_s")])
        try:
            return thunk()
        finally:
            self.stop(totals, key, began)


@dataclass
class _StepRecord:
    """What one update produced for logs and rank timing."""

    out: Optional[Dict[str, Any]] = None
    loss: Optional[torch.Tensor] = None
    loss_value: Optional[float] = None
    batch_wait_s: float = 0.0
    extra_timing: Dict[str, float] = field(default_factory=dict)
    timings: Dict[str, float] = field(default_factory=dict)
    skip_counts: Dict[str, float] = field(default_factory=dict)


class _MicroSteps:
    """Gradient accumulation over ``grad_accum`` micro-batches."""

    def __init__(self, run: "_Run") -> None:
        self.run_ = run

    def __call__(self, step: int, batches: Iterator[Any], *, want_rank_timing: bool) -> _StepRecord:
        r = self.run_
        s = r.settings
        rec = _StepRecord()
        prof = r.profiler
        count = s.grad_accum
        prefetching = r.on_cuda and s.prefetch_batches > 0
        can_defer_sync = hasattr(r.model, "no_sync")
        graphed = r.graphed_step if count == 1 else None
        for micro in range(count):
            defer = r.model.no_sync() if can_defer_sync and micro < count - 1 else nullcontext()
            cast = r.autocast() if not s.autocast_in_step_fn else nullcontext()
            # In graph mode forward and backward always run on the graph's own stream (eager updates too),
            # so the autograd nodes of the parameters are made on the stream the capture uses.
            side = graphed.on_side_stream() if graphed is not None else nullcontext()
            with side:
                out, loss = self._one(r, step, micro, count, batches, rec, graphed, defer, cast, prefetching,
                                      want_rank_timing)
            part = loss.detach()
            rec.loss = part if rec.loss is None else rec.loss + part
            rec.out = out
        return rec

    @staticmethod
    def _one(r, step, micro, count, batches, rec, graphed, defer, cast, prefetching, want_rank_timing):
        """One micro-batch: fetch, step_fn, backward (or the captured graph). Returns (output, loss)."""

        s, prof = r.settings, r.profiler
        backward_done = False
        with defer, cast:
            r.micro_position = (micro, "fetch")
            began = prof.start("batch_wait")
            batch = next(batches) if prefetching else to_device(next(batches), r.device)
            rec.batch_wait_s += prof.stop(rec.timings, "profile_loop_batch_wait_time_s", began)
            for k, v in _skip_counters(batch).items():
                rec.skip_counts[k] = rec.skip_counts.get(k, 0.0) + v
            r.micro_position = (micro, "step_fn")
            if graphed is not None and graphed.wants(batch):
                def forward(b):
                    o = _checked(r.step_fn(r.model, b, r.step_ctx(step)))
                    lo = o["loss"] / count
                    return o, lo, r.scaler.scale(lo)

                out, loss = prof.run(rec.timings, "profile_loop_step_fn_time_s", lambda: graphed.run(batch, forward))
                backward_done = True
            else:
                out = _checked(prof.run(rec.timings, "profile_loop_step_fn_time_s",
                                        lambda: r.step_fn(r.model, batch, r.step_ctx(step))))
                if graphed is not None:
                    graphed.note_eager()
                loss = out["loss"] / count
            if want_rank_timing and isinstance(out, Mapping):
                for key in s.rank_timing_extra_keys:
                    if out.get(key) is not None:
                        v = out[key]
                        rec.extra_timing[key] = rec.extra_timing.get(key, 0.0) + float(
                            v.detach() if isinstance(v, torch.Tensor) else v)
        r.micro_position = (micro, "backward")
        if not backward_done:
            prof.run(rec.timings, "profile_loop_backward_time_s", lambda: r.scaler.scale(loss).backward())
        return out, loss


class _StopControl:
    """Per-update agreement on stopping (evacuation, GPU health) and what an agreed stop does."""

    def __init__(self, run: "_Run") -> None:
        self.run_ = run

    def reconcile(self, step: int) -> None:
        r = self.run_
        r.health.update_step(step)
        local = r.health.failures()
        evacuate, unhealthy = r.evacuation.reconcile_requests(bool(local))
        r.evacuation_requested = evacuate
        r.ctx["evacuation_requested"] = evacuate
        if unhealthy:
            everyone = [local]
            if dist_lib.is_initialized():
                everyone = [None] * r.world_size
                torch.distributed.all_gather_object(everyone, local)
            self._stop_for_health(step, [f for per_rank in everyone for f in per_rank])

    def _stop_for_health(self, step: int, failures: list) -> None:
        r = self.run_
        h = r.health
        h.close()
        completed = step + 1
        bad_nodes = h.bad_nodes_from_failures(failures)
        metrics = {"gpu_health": {"event": "gpu_health_shutdown", "failures": failures, "bad_nodes": bad_nodes,
                                  "slurm_action": h.slurm_action, "slurm_disabled": h.slurm_disabled}}
        path, ckpt = r.checkpoint(completed, next_step=completed, metrics=metrics, gather_rng=True, announce=False)
        r.final_ckpt = ckpt
        dist_lib.barrier()
        if r.is_rank0:
            r.emit("on_checkpoint", path, ckpt, r.step_ctx(completed))
            summary = h.write_failure_summary(step=completed, failures=failures, checkpoint_path=path)
            print(f"[gpu-health] FAIL step={step} {summarize_failures_for_stdout(failures)}", flush=True)
            print(f"[gpu-health] checkpoint={path} summary={summary} slurm_action={h.slurm_action} "
                  f"bad_nodes={','.join(bad_nodes)}", flush=True)
        dist_lib.barrier()
        if r.is_rank0:
            results = h.perform_slurm_recovery(failures)
            if results:
                print(f"[gpu-health] slurm_results={json.dumps(results, sort_keys=True)}", flush=True)
        elif os.environ.get("SLURM_JOB_ID") and not h.slurm_disabled and h.slurm_action in {"requeue", "cancel"}:
            time.sleep(30.0)  # rank 0 mutates the Slurm job before the job is torn down
        raise SystemExit(h.exit_code)


class _OomGuard:
    """Opt-in survival of CUDA OOMs raised while a step fetches, runs ``step_fn`` or backward."""

    def __init__(self, run: "_Run", settings: oom_lib.OomRecoverySettings) -> None:
        self.run_ = run
        self.settings = settings
        self.catches: tuple = (oom_lib.OutOfMemoryError,) if settings.enabled else ()
        self.skipped: set = set()

    def load_records(self, start: int) -> None:
        """Learn the steps earlier attempts recorded as OOM (rank 0 reads, everyone receives)."""

        r = self.run_
        steps = sorted(oom_lib.recorded_steps(r.keeper.store)) if r.is_rank0 else None
        if r.world_size > 1 and dist_lib.is_initialized():
            box = [steps]
            torch.distributed.broadcast_object_list(box, src=0)
            steps = box[0]
        self.skipped = set(steps or ())
        upcoming = [s for s in sorted(self.skipped) if start <= s < r.settings.max_steps]
        if upcoming and r.is_rank0:
            shown = ", ".join(map(str, upcoming[:20])) + (", ..." if len(upcoming) > 20 else "")
            print(f"[oom] {len(upcoming)} step(s) recorded as OOM-skipped by earlier attempts will be skipped: {shown}",
                  flush=True)

    def record(self, step: int, exc: BaseException) -> Dict[str, Any]:
        r = self.run_
        micro, phase = r.micro_position
        verdict = oom_lib.decide(self.settings, self.skipped, step, distributed=r.world_size > 1,
                                 during_fetch=phase == "fetch")
        memory, summary = oom_lib.memory_report(r.device)
        rec = {"v": 1, "step": step, "rank": r.rank, "world_size": r.world_size, "phase": phase,
               "micro_step": micro, "grad_accum": r.settings.grad_accum, "action": verdict.action,
               "reason": verdict.reason, "consecutive": verdict.consecutive,
               "max_consecutive": self.settings.max_consecutive, "skipped_total": verdict.skipped_total,
               "error_type": type(exc).__name__, "message": oom_lib.short_message(exc), "memory": memory,
               "memory_summary": summary, "wall_time": time.time()}
        print(oom_lib.format_record(rec), flush=True)
        return rec

    def recover(self, step: int, batches: Iterator[Any], rec: Dict[str, Any]) -> bool:
        r = self.run_
        r.optimizer.zero_grad(set_to_none=True)
        oom_lib.release_memory(r.device)
        oom_lib.write_record(r.keeper.store, rec)  # durable before anything else can fail
        self.skipped.add(step)
        r.emit("on_oom", rec, r.step_ctx(step))
        if r.world_size > 1:
            print(f"[oom] rank={r.rank} exiting with code {OOM_RESTART_EXIT_CODE}; resubmit with resume=auto to "
                  "continue from the last checkpoint", flush=True)
            raise SystemExit(OOM_RESTART_EXIT_CODE)
        consumed = 0 if rec["phase"] == "fetch" else int(rec["micro_step"]) + 1
        if rec["phase"] != "fetch" and not self._discard(batches, r.settings.grad_accum - consumed):
            return False
        r.step_scheduler()
        if rec["action"] == oom_lib.RESTART:
            completed = step + 1
            path, r.final_ckpt = r.checkpoint(completed, next_step=completed, gather_rng=True, announce=False)
            r.emit("on_checkpoint", path, r.final_ckpt, r.step_ctx(completed))
            print(f"[oom] checkpoint={path} next_step={completed}; exiting with code {OOM_RESTART_EXIT_CODE} so a "
                  "resubmit starts with a fresh CUDA allocator", flush=True)
            raise SystemExit(OOM_RESTART_EXIT_CODE)
        return r.after_update(step, {})

    def replay_skip(self, step: int, batches: Iterator[Any]) -> bool:
        r = self.run_
        if not self._discard(batches, r.settings.grad_accum):
            return False
        r.step_scheduler()
        if r.is_rank0:
            print(f"[oom] step={step} skipped: recorded as OOM by an earlier attempt", flush=True)
        return r.after_update(step, {})

    @staticmethod
    def _discard(batches: Iterator[Any], n: int) -> bool:
        for _ in range(n):
            try:
                next(batches)
            except StopIteration:
                return False
        return True


# ----------------------------------------------------------------------------- the run


class _Run:
    """One call of ``training_loop`` (not public API)."""

    def __init__(self, *, model, dataset, step_fn, optimizer, scheduler, train_cfg, config_json, checkpoint_dict,
                 eval_dataset, eval_fn, prepare_batch_fn, hooks, resume, auto_resume_path, evacuation) -> None:
        train_cfg, config_json = _split_root_config(train_cfg, config_json)
        self.train_cfg = train_cfg
        self.settings = s = LoopSettings.from_cfg(train_cfg)
        self.ema_settings = EmaSettings.from_cfg(train_cfg)
        self.step_fn, self.optimizer, self.scheduler = step_fn, optimizer, scheduler
        self.dataset, self.eval_dataset, self.eval_fn = dataset, eval_dataset, eval_fn
        self.prepare_batch_fn = prepare_batch_fn
        self.hooks = hooks
        all_rank_hooks = bool(hooks and hooks.get("on_checkpoint_all_ranks"))
        if s.checkpoint_async and all_rank_hooks:
            raise ValueError("All-rank checkpoint hooks require synchronous publication")
        self.checkpoint_dict = checkpoint_dict
        self.resume_mode = str(resume if resume is not None else config_lib.get(train_cfg, "resume", "none")).lower()
        if self.resume_mode not in {"none", "auto"}:
            raise ValueError("resume must be 'none' or 'auto'")
        if auto_resume_path is not None and self.resume_mode != "auto":
            raise ValueError("auto_resume_path requires resume='auto'")
        if auto_resume_path is not None and checkpoint_dict is None:
            raise ValueError("auto_resume_path requires a preloaded checkpoint")
        self.auto_resume_path = auto_resume_path
        if isinstance(evacuation, EvacuationController):
            self.evacuation = evacuation
        elif isinstance(evacuation, bool):
            self.evacuation = EvacuationController(evacuation)
        else:
            self.evacuation = EvacuationController(bool(config_lib.get(train_cfg, "evacuation_enabled", False)),
                                                   signal_name=config_lib.get(train_cfg, "evacuation_signal", "USR1"))
        self.evacuation_requested = False
        self.micro_position: Tuple[int, str] = (0, "fetch")
        self.freezer = WarmFreeze()

        self.device = ensure_process_device(get_device(train_cfg))
        model.to(self.device)
        self.model: nn.Module = model
        self.rank, self.world_size, self.is_rank0 = dist_lib.rank(), dist_lib.world_size(), dist_lib.rank0()
        self.on_cuda = getattr(self.device, "type", "cpu") == "cuda"
        self.keeper = CheckpointKeeper(location=s.checkpoint_dir, keep_last_k=s.keep_last_k,
                                       background=s.checkpoint_async, is_rank0=self.is_rank0,
                                       world_size=self.world_size, emit=self.emit, has_all_rank_hooks=all_rank_hooks)
        self.scaler = make_scaler(s.amp_mode)
        self.cfg_json = config_lib.as_dict(config_json if config_json is not None else train_cfg)
        self.ctx: Dict[str, Any] = {
            "device": self.device, "rank": self.rank, "world_size": self.world_size, "autocast": self.autocast,
            "scaler": self.scaler, "config": self.cfg_json, "config_json": self.cfg_json, "train_cfg": train_cfg,
            "model": self.model, "evacuation_requested": False, "resume_mode": self.resume_mode,
            "auto_resume_selected": False,
        }
        self.ema: Optional[EMA] = None
        self.ema_dual: List[EMA] = []
        self._ema_in_optimizer = False
        self.final_ckpt: Optional[Dict[str, Any]] = checkpoint_dict
        self.health = BackgroundGpuHealth(device=self.device, out_dir=s.out_dir, rank=self.rank,
                                          world_size=self.world_size)
        self.profiler = _Profiler(s, self.on_cuda, self.device)
        self.gate = GradientGate(max_norm=s.grad_clip_norm, check_every=s.nonfinite_grad_check_every,
                                 scaler=self.scaler, profile=lambda key, thunk: thunk())
        self.graphed_step: Optional[GraphedStep] = None
        if s.cuda_graph_step and self.on_cuda and self.world_size == 1 and s.grad_accum == 1:
            self.graphed_step = GraphedStep(model, warmup=s.cuda_graph_warmup)
        self.micro_steps = _MicroSteps(self)
        self.stops = _StopControl(self)
        self.oom = _OomGuard(self, oom_lib.OomRecoverySettings.from_cfg(train_cfg))

    # ------------------------------------------------------------------ shared helpers
    def emit(self, event: str, *args, suppress_exceptions: bool = True, **kwargs) -> None:
        hooks_lib.emit(self.hooks, event, *args, suppress_exceptions=suppress_exceptions, **kwargs)

    def autocast(self):
        return autocast_context(self.settings.amp_mode, self.device)

    def step_ctx(self, step: int) -> Dict[str, Any]:
        return {**self.ctx, "step": step, "optimizer": self.optimizer, "ema": self.ema}

    def unwrapped(self) -> nn.Module:
        return getattr(self.model, "module", self.model)

    def checkpoint(self, step: int, *, next_step: int, metrics=None, gather_rng: bool = False, announce: bool = True,
                   background: bool = False) -> Tuple[str, Dict[str, Any]]:
        """Every rank collects the checkpoint; rank 0 publishes it. Returns (path, dict) on every rank."""

        ckpt = self.keeper.collect(step=step, next_step=next_step, module=self.unwrapped(), optimizer=self.optimizer,
                                   scheduler=self.scheduler, scaler=self.scaler, config=self.cfg_json, ema=self.ema,
                                   dual=self.ema_dual, oom_skipped=self.oom.skipped, metrics=metrics,
                                   gather_rng=gather_rng)
        if not self.is_rank0:
            return self.keeper.path_of(step), ckpt
        tell = (lambda path: self.emit("on_checkpoint", path, ckpt, self.step_ctx(step))) if announce else None
        return self.keeper.publish(step, ckpt, announce=tell, background=background), ckpt

    def step_scheduler(self) -> None:
        if self.scheduler is not None and self.settings.scheduler_step_policy == "step":
            try:
                self.scheduler.step()
            except TypeError:
                pass  # a scheduler that steps on a metric after eval

    # ------------------------------------------------------------------ setup
    def _shard_inputs(self) -> None:
        s = self.settings
        mode = shard_mode(s.shard_dataset_enabled, s.shard_dataset_mode, "shard_dataset")
        eval_mode = shard_mode(s.shard_eval_dataset_enabled, s.shard_eval_dataset_mode, "shard_eval_dataset")
        if not s.ddp_enabled:
            return
        if mode is not None:
            self.dataset = shard_dataset(self.dataset, rank=self.rank, world_size=self.world_size, mode=mode)
        if self.eval_dataset is not None and eval_mode is not None:
            self.eval_dataset = shard_dataset(self.eval_dataset, rank=self.rank, world_size=self.world_size,
                                              mode=eval_mode)
        if s.warn_unsharded and self.is_rank0:
            warn_if_unsharded(self.dataset, enabled=True, name="train dataset")
            warn_if_unsharded(self.eval_dataset, enabled=True, name="eval dataset")

    def _compile(self) -> None:
        """Opt-in ``torch.compile`` of the model before data-parallel wrapping (never on the native hot path)."""

        setting = config_lib.get(self.train_cfg, "compile", None)
        if not setting:
            return
        kwargs: Dict[str, Any] = {}
        enabled, preset = True, None
        if isinstance(setting, Mapping):
            enabled, preset = bool(setting.get("enabled", True)), setting.get("preset")
            kwargs = {k: v for k, v in setting.items() if k not in ("enabled", "preset")}
        elif isinstance(setting, str):
            preset = setting
        elif isinstance(setting, bool):
            enabled = setting
        if not enabled:
            return
        preset = None if preset is None else str(preset)
        if preset is not None:
            kwargs.setdefault("mode", "max-autotune" if preset.lower() in _COMPILE_FULL else preset)
        wraps_only = preset is not None and preset.lower() in _COMPILE_WRAPS_ONLY
        undo: List[Callable[[], None]] = []
        was_enabled = flags_lib.get_compile_wrap_enabled()
        if wraps_only:
            undo += self._dynamo_skip_unwrapped()
        else:
            flags_lib.set_compile_wrap_enabled(False)
            undo += self._strip_compile_wraps()
        try:
            prepare_compile_backend()
            self.model = torch.compile(self.model, **kwargs)
            self.ctx["model"] = self.model
        except Exception as exc:
            for restore in undo:
                restore()
            flags_lib.set_compile_wrap_enabled(was_enabled)
            if self.is_rank0:
                warnings.warn(f"torch.compile failed; falling back to eager: {exc}", RuntimeWarning)

    def _dynamo_skip_unwrapped(self) -> List[Callable[[], None]]:
        undo: List[Callable[[], None]] = []

        def walk(module: nn.Module, covered: bool) -> None:
            covered = covered or isinstance(getattr(type(module), "forward", None), flags_lib.compile_wrap)
            if module is not self.model and not covered:
                original = module.forward
                module.forward = torch._dynamo.disable(module.forward)
                undo.append(lambda m=module, f=original: setattr(m, "forward", f))
            for child in module.children():
                walk(child, covered)

        walk(self.model, False)
        return undo

    def _strip_compile_wraps(self) -> List[Callable[[], None]]:
        undo: List[Callable[[], None]] = []
        for cls in {type(m) for m in self.model.modules()}:
            wrapped = getattr(cls, "forward", None)
            if isinstance(wrapped, flags_lib.compile_wrap):
                setattr(cls, "forward", wrapped.function)
                undo.append(lambda c=cls, w=wrapped: setattr(c, "forward", w))
        return undo

    def _wrap_data_parallel(self) -> None:
        s = self.settings
        if not (s.ddp_enabled and self.world_size > 1):
            return
        assert dist_lib.is_initialized()
        if self.on_cuda and str(torch.distributed.get_backend()).lower() == "nccl":
            from .parallel.ddp import DataParallel

            owners, shard_rest = {}, False
            commit = getattr(self.optimizer, "kb_commit_gradient_plan", None)
            if s.comm_transport.lower() in ("fused", "p2p") and callable(commit):
                owners, shard_rest = commit(self.world_size)
            self.model = DataParallel(self.model, bucket_cap_mb=s.bucket_caps_mb(),
                                      broadcast_buffers=s.ddp_broadcast_buffers, transport=s.comm_transport,
                                      find_unused_parameters=s.find_unused_parameters, owners=owners,
                                      shard_rest=shard_rest)
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
            if self.on_cuda:
                kw["device_ids"] = [torch.cuda.current_device()]
            self.model = DistributedDataParallel(self.model, **kw)
        self.ctx["model"] = self.model

    def _pick_resume(self) -> Optional[str]:
        if self.resume_mode != "auto":
            return None
        if self.checkpoint_dict is not None:
            if self.auto_resume_path is None:
                return None
            self.ctx["auto_resume_selected"] = True
            return self.auto_resume_path
        found = checkpoint_lib.resolve_auto_resume(self.keeper.store)
        if found is None:
            return None
        path, self.checkpoint_dict = found
        self.ctx["auto_resume_selected"] = True
        return path

    def _resume(self) -> int:
        ckpt = self.checkpoint_dict
        if not (ckpt and isinstance(ckpt, dict)):
            return 0
        start = restore_training_state(ckpt, model=self.model, optimizer=self.optimizer, scheduler=self.scheduler,
                                       scaler=self.scaler, rank=self.rank)
        self.ema, self.ema_dual = restore_ema(self.unwrapped(), self.ema_settings, ckpt.get("ema"),
                                              ckpt.get("ema_dual"))
        return start

    def _batches(self) -> Iterator[Any]:
        s = self.settings
        if self.on_cuda and s.prefetch_batches > 0:
            return prefetch(iter(self.dataset), self.device, prefetch=s.prefetch_batches,
                            prepare_fn=self.prepare_batch_fn, threaded=s.prefetch_threaded,
                            pipeline=s.prefetch_pipeline)
        return iter(self.dataset)

    # ------------------------------------------------------------------ one update
    def _update_parameters(self, step: int, rec: _StepRecord) -> None:
        prof, t = self.profiler, rec.timings

        def wait_for_ema_snapshots() -> None:
            for e in ([self.ema] if self.ema is not None else []) + self.ema_dual:
                e.wait_before_param_mutation()

        prof.run(t, "profile_loop_ema_wait_time_s", wait_for_ema_snapshots)
        self._hand_ema_to_optimizer(step)
        prof.run(t, "profile_loop_optimizer_step_time_s", lambda: self.scaler.step(self.optimizer))
        # The gate's outcome: read now that the step is enqueued (a rejected step was skipped on the device
        # and raises here under clipping, before the EMA, the scheduler or any hook sees it).
        clip = self.gate.finish(self.model, self.optimizer)
        if clip:
            rec.out = {} if rec.out is None else rec.out
            rec.out.update(clip)
        prof.run(t, "profile_loop_scaler_update_time_s", self.scaler.update)
        prof.run(t, "profile_loop_ema_update_time_s", lambda: self._update_ema(step))
        prof.run(t, "profile_loop_scheduler_time_s", self.step_scheduler)

    def _hand_ema_to_optimizer(self, step: int) -> None:
        """Let a fused single-process optimizer apply this step's EMA update inside its own kernels."""

        self._ema_in_optimizer = False
        if self.ema is None or self.ema_dual or isinstance(self.scaler, GradScaler) or not self.ema.fusable():
            return
        target = self.optimizer if getattr(self.optimizer, "kb_fused", False) else getattr(self.optimizer, "inner",
                                                                                           None)
        if target is None or not getattr(target, "kb_fused", False):
            return
        if self.world_size > 1 and getattr(target, "_distributed", False):
            return
        es = self.ema_settings
        target.kb_ema = self.ema.begin_fused_update(self.unwrapped(), None if es.profile == "power"
                                                    else es.warmed_decay(step))
        self._ema_in_optimizer = True

    def _update_ema(self, step: int) -> None:
        es = self.ema_settings
        keeps_ema = self.is_rank0 or self.keeper.all_rank_hooks
        module = self.unwrapped()
        if keeps_ema and self.ema is None and es.enabled:
            self.ema = EmaBuilder(es).single(module)
        if keeps_ema and not self.ema_dual and es.dual.enabled:
            self.ema_dual = EmaBuilder(es).pair(module)
        if self.ema is not None and not self._ema_in_optimizer:
            if es.profile == "power":
                self.ema.update(module)
            else:
                self.ema.update(module, decay=es.warmed_decay(step))
        for e in self.ema_dual:
            e.update(module)
        self._ema_in_optimizer = False

    def _logs(self, step: int, rec: _StepRecord, seconds: float) -> Tuple[Optional[Dict[str, Any]], Dict[str, Any]]:
        lr = get_lr(self.optimizer)
        loss: Any = rec.loss_value if rec.loss_value is not None else (rec.loss if rec.loss is not None else 0.0)
        minimal: Dict[str, Any] = {"loss": loss, "lr": lr, "step_time_s": seconds, "step": step}
        if not (self.is_rank0 and step % self.settings.log_every == 0):
            return None, minimal
        value = float(rec.loss_value if rec.loss_value is not None else (rec.loss if rec.loss is not None else 0.0))
        rec.loss_value = value
        extras = {k: (float(v.detach()) if isinstance(v, torch.Tensor) else v)
                  for k, v in (rec.out or {}).items() if k != "loss"}
        profiled = {k: float(v) for k, v in rec.timings.items() if k.startswith("profile_loop_")}
        full = {"loss": value, "lr": lr, "step_time_s": seconds, **rec.skip_counts, **extras, **profiled, "step": step}
        return full, full

    def _rank_timing(self, step: int, rec: _StepRecord, seconds: float) -> None:
        mine: Dict[str, Any] = {"rank": self.rank, "batch_wait_s": float(rec.batch_wait_s),
                                "step_compute_s": float(max(0.0, seconds - rec.batch_wait_s)),
                                "total_step_s": float(seconds)}
        for key in self.settings.rank_timing_extra_keys:
            mine[key] = float(rec.extra_timing.get(key, rec.timings.get(key, 0.0)))
        everyone: list = [None] * self.world_size
        torch.distributed.all_gather_object(everyone, mine)
        if self.is_rank0:
            print(_rank_timing_line([e for e in everyone if isinstance(e, dict)], step,
                                    self.settings.rank_timing_extra_keys))

    def _one_update(self, step: int, batches: Iterator[Any]) -> bool:
        if step in self.oom.skipped:
            return self.oom.replay_skip(step, batches)
        s, prof = self.settings, self.profiler
        began = prof.start()
        timer = self._start_device_timer()
        prelude: Dict[str, float] = {}

        def reset() -> None:
            self.model.train()
            self.optimizer.zero_grad(set_to_none=True)

        prof.run(prelude, "profile_loop_setup_zero_grad_time_s", reset)
        want_timing = (s.ddp_enabled and self.world_size > 1 and s.rank_timing_every > 0
                       and step % s.rank_timing_every == 0)
        oom_rec = None
        try:
            rec = self.micro_steps(step, batches, want_rank_timing=want_timing)
        except StopIteration:
            return False
        except self.oom.catches as exc:
            oom_rec = self.oom.record(step, exc)
            if oom_rec["action"] == oom_lib.FAIL:
                raise
        if oom_rec is not None:
            return self.oom.recover(step, batches, oom_rec)
        for k, v in prelude.items():
            rec.timings[k] = rec.timings.get(k, 0.0) + v

        self.gate.profile = lambda key, thunk: prof.run(rec.timings, key, thunk)
        self.gate.begin(self.model, self.optimizer, step, self.on_cuda)
        self._update_parameters(step, rec)
        if s.scalarize_loss_every_step and rec.loss is not None:
            # Read once per update, after the optimizer step is enqueued (the sum of the micro-step losses):
            # a read after each micro-step would stall the GPU while the host enqueues the next one.
            rec.loss_value = float(rec.loss)

        prof.barrier()
        seconds = time.perf_counter() - began
        device_ms = self._stop_device_timer(timer)
        if want_timing:
            self._rank_timing(step, rec, seconds)
        mark = prof.start("log_build")
        full, minimal = self._logs(step, rec, seconds)
        if device_ms is not None:
            for d in (minimal, full):
                if d is not None:
                    d["step_device_ms"] = device_ms
        built = prof.stop(rec.timings, "profile_loop_log_build_time_s", mark)
        if s.profile_step_timing:
            for d in (minimal, full):
                if d is not None:
                    d["profile_loop_log_build_time_s"] = built
        mark = prof.start("log_emit")
        ctx = self.step_ctx(step)
        self.emit("on_update_end", minimal, ctx)
        if full is not None:
            self.emit("on_log", full, ctx)
        self.emit("on_step_end", minimal, ctx)
        prof.stop(rec.timings, "profile_loop_log_emit_time_s", mark)
        self.freezer.update()
        return self.after_update(step, rec.timings)

    def _start_device_timer(self):
        if not (self.settings.device_timing and self.on_cuda):
            return None
        pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        pair[0].record()
        return pair

    @staticmethod
    def _stop_device_timer(pair) -> Optional[float]:
        if pair is None:
            return None
        pair[1].record()
        pair[1].synchronize()
        return float(pair[0].elapsed_time(pair[1]))

    def after_update(self, step: int, timings: Dict[str, float]) -> bool:
        """Stop agreement, eval, periodic checkpoint -- after every update (also skipped ones)."""

        s, prof = self.settings, self.profiler
        prof.run(timings, "profile_loop_health_check_time_s", lambda: self.stops.reconcile(step))
        prof.run(timings, "profile_loop_eval_time_s", lambda: self._maybe_eval(step))
        if self.evacuation_requested:
            return True
        mark = prof.start("checkpoint")
        at = step + int(s.intervals_use_completed_steps)
        terminal_next = s.intervals_use_completed_steps and at == s.max_steps
        if at > 0 and at % s.ckpt_every == 0 and not terminal_next:
            path, ckpt = self.checkpoint(at, next_step=step + 1, gather_rng=True, background=s.checkpoint_async)
            if self.is_rank0:
                self.final_ckpt = ckpt
            if not s.checkpoint_async:
                dist_lib.barrier()  # peers wait until rank 0 has published
            self.keeper.all_rank_hooks_run(path, ckpt, self.step_ctx(at))
        self.keeper.poll()
        prof.stop(timings, "profile_loop_checkpoint_time_s", mark)
        return True

    def _maybe_eval(self, step: int) -> None:
        s = self.settings
        if self.eval_fn is None or self.eval_dataset is None or s.eval_every <= 0:
            return
        at = step + int(s.intervals_use_completed_steps)
        if (at == 0 and not s.eval_at_step_zero) or at % s.eval_every != 0:
            return
        if self.ema is not None and self.ema_settings.eval_with_ema:
            module = self.unwrapped()
            self.ema.store(module)
            self.ema.copy_to(module)
            try:
                metrics = self.eval_fn(self.model, self.eval_dataset, self.step_ctx(step))
            finally:
                self.ema.restore(module)
        else:
            metrics = self.eval_fn(self.model, self.eval_dataset, self.step_ctx(step))
        if self.scheduler is not None and s.scheduler_step_policy == "eval":
            self.scheduler.step(metrics.get("val_loss", None))
        if self.is_rank0:
            self.emit("on_eval_end", metrics, self.step_ctx(step))

    # ------------------------------------------------------------------ the whole run
    def execute(self) -> Dict[str, Any]:
        batches: Optional[Iterator[Any]] = None
        try:
            self.evacuation.install()
            if self.evacuation.already_evacuated:
                print("[evacuation] run already evacuated; exiting before training", flush=True)
                raise SystemExit(EVACUATION_EXIT_CODE)
            self.health.start()
            self._shard_inputs()
            resume_path = self._pick_resume()
            self.emit("on_train_start", self.ctx, suppress_exceptions=False)
            self._compile()
            self._wrap_data_parallel()
            if self.is_rank0:
                total, trainable = _parameter_counts(self.model)
                print(f"[training] Model parameters — total: {total:,} | trainable: {trainable:,} | "
                      f"frozen: {total - trainable:,}")
            start = self._resume()
            if self.oom.settings.enabled:
                self.oom.load_records(start)
            if resume_path is not None and self.is_rank0:
                self.emit("on_resume_checkpoint", resume_path, self.checkpoint_dict, self.step_ctx(start))
            batches = self._batches()
            done, stopped = start, False
            for step in range(start, self.settings.max_steps):
                if not self._one_update(step, batches):
                    break
                done = step + 1
                if self.evacuation_requested:
                    stopped = True
                    break
            self._finish(done, stopped)
        except Exception as exc:
            self.emit("on_exception", exc, self.ctx)
            raise
        finally:
            with ExitStack() as cleanup:
                closer = getattr(batches, "close", None)
                if callable(closer):
                    cleanup.callback(closer)
                cleanup.callback(self.keeper.close)
                cleanup.callback(self.evacuation.uninstall)
                cleanup.callback(self.health.close)
        assert self.final_ckpt is not None
        return self.final_ckpt

    def _finish(self, done: int, stopped: bool) -> None:
        """Last stop agreement, terminal checkpoint (cursor == step), evacuation exit if asked."""

        self.health.close()
        self.stops.reconcile(done - 1)
        stopped = stopped or self.evacuation_requested
        path, self.final_ckpt = self.checkpoint(done, next_step=done, gather_rng=True, announce=False)
        if dist_lib.is_initialized():
            dist_lib.barrier()
        if self.is_rank0:
            self.emit("on_checkpoint", path, self.final_ckpt, self.step_ctx(done))
        self.keeper.all_rank_hooks_run(path, self.final_ckpt, self.step_ctx(done))
        if stopped:
            if self.is_rank0:
                self.emit("on_evacuation", path, self.final_ckpt, self.step_ctx(done))
            self.emit("on_train_end", self.ctx)
            if dist_lib.is_initialized():
                dist_lib.barrier()
            self.evacuation.mark_evacuated()
            raise SystemExit(EVACUATION_EXIT_CODE)
        self.emit("on_train_end", self.ctx)
