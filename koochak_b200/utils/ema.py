"""Exponential moving average (EMA) of a model's trainable parameters.

(behaviour of reference koochak/utils/ema.py:6-327; the state-dict keys are
the checkpoint format shared with it)

An ``EMA`` is three parts:

* ``_Schedule`` -- which decay an update uses. ``constant``: d, raised to the
  number of steps since the previous update when updates are thinned
  (``update_every`` > 1); ``power``: ((t - elapsed) / t) ** (gamma + 1), the
  EDM2 power profile (gamma may be given through its relative width
  ``srel``). It also owns the counters saved in checkpoints.
* the shadows -- fp32 copies keyed by parameter name, either on the
  parameters' GPU (updated by one native multi-tensor kernel, or folded into
  a fused optimizer's own update pass through ``begin_fused_update``), or on
  the host (the reference's default, ``offload_to_cpu=True``);
* ``_HostMirror`` -- for host shadows: after each update a snapshot of the
  parameters is copied device-to-host on a side stream into pinned staging
  buffers, and a one-thread worker applies the math once the copy lands.
  ``wait_before_param_mutation`` blocks until the snapshot no longer reads
  the live parameters, so the optimizer may then overwrite them.
"""

from __future__ import annotations

import math
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from typing import Dict, Iterator, List, Optional, Tuple

import torch

__all__ = ["EMA"]


def _srel_of_gamma(gamma: float) -> float:
    g = float(gamma)
    return math.sqrt(g + 1.0) / ((g + 2.0) * math.sqrt(g + 3.0))


def _gamma_of_srel(srel: float) -> float:
    """Invert ``_srel_of_gamma`` (monotone decreasing) by bisection in log space."""

    goal = max(1e-9, float(srel))
    lo, hi = 1e-6, 1e6
    for _ in range(64):
        mid = math.sqrt(lo * hi)
        lo, hi = (mid, hi) if _srel_of_gamma(mid) > goal else (lo, mid)
    return 0.5 * (lo + hi)


@dataclass
class _Schedule:
    decay: float
    profile: str
    gamma: Optional[float]
    update_every: int
    num_updates: int = 0
    step_counter: int = 0
    last_update: int = 0

    def advance(self, override: Optional[float]) -> Optional[float]:
        """Count one step; the decay to apply now, or None when thinning skips this step."""

        self.step_counter += 1
        if self.step_counter % self.update_every:
            return None
        elapsed = max(1, self.step_counter - self.last_update)
        if self.profile == "power" and override is None:
            g = 6.94 if self.gamma is None else float(self.gamma)
            t = max(1.0, float(self.step_counter))
            d = (max(0.0, t - elapsed) / t) ** (g + 1.0)
        else:
            d = float(self.decay if override is None else override)
            if self.profile == "constant":
                d = d ** elapsed
        self.num_updates += 1
        return float(d)

    def mark_applied(self) -> None:
        self.last_update = self.step_counter


class _HostMirror:
    """Device-to-host snapshots on a side stream and the shadow math on one worker thread."""

    def __init__(self, device: torch.device, shadows: Dict[str, torch.Tensor], pin: bool) -> None:
        self.device = device
        self.staging = {k: torch.empty_like(v, device="cpu", pin_memory=pin) for k, v in shadows.items()}
        with torch.cuda.device(device):
            self.stream = torch.cuda.Stream(device=device)
        self.pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="koochak-ema")
        self.copied: Optional[torch.cuda.Event] = None
        self.job: Optional[Future] = None

    def snapshot(self, params: Iterator[Tuple[str, torch.Tensor]], dtype: torch.dtype,
                 apply: "callable") -> None:
        with torch.cuda.device(self.device):
            produced = torch.cuda.Event(blocking=False)
            produced.record(torch.cuda.current_stream(self.device))
            landed = torch.cuda.Event(blocking=False)
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(produced)
                for name, p in params:
                    src = p.detach()
                    self.staging[name].copy_(src if src.dtype is dtype else src.to(dtype=dtype), non_blocking=True)
                landed.record(self.stream)
        self.copied = landed
        self.job = self.pool.submit(lambda: (landed.synchronize(), apply(self.staging)))

    def release_params(self) -> None:
        if self.copied is not None:
            if not torch.cuda.is_available():
                raise RuntimeError("EMA has a pending CUDA snapshot but CUDA is not available on this process")
            self.copied.synchronize()
            self.copied = None

    def drain(self) -> None:
        self.release_params()
        if self.job is not None:
            job, self.job = self.job, None
            job.result()


class EMA:
    def __init__(self, model: torch.nn.Module, decay: float = 0.999, *, dtype: torch.dtype = torch.float32,
                 profile: str = "constant", gamma: Optional[float] = None, srel: Optional[float] = None,
                 update_every: int = 1, offload_to_cpu: bool = True, pin_memory: bool = True,
                 compensate_update_every: bool = True) -> None:
        if not 0.0 < float(decay) < 1.0:
            raise ValueError("EMA decay must be in (0, 1)")
        kind = (profile or "constant").lower()
        if kind not in ("constant", "power"):
            raise ValueError(f"Unsupported EMA profile: {kind}")
        if gamma is None and srel is not None:
            gamma = _gamma_of_srel(float(srel))
        self._sched = _Schedule(float(decay), kind, None if gamma is None else float(gamma), max(1, int(update_every)))
        self.dtype = dtype
        self.offload = bool(offload_to_cpu)
        self.pin_memory = bool(pin_memory)
        # Thinned updates are always compensated; the flag stays in the checkpoint format.
        self.compensate_update_every = True
        self.shadow: Dict[str, torch.Tensor] = {}
        self._saved: Optional[Dict[str, torch.Tensor]] = None
        copy_device = None
        for name, p in self._tracked(model):
            self.shadow[name] = p.detach().to(device="cpu" if self.offload else p.device, dtype=dtype).clone()
            if self.offload and p.is_cuda and copy_device is None:
                copy_device = p.device
        self._mirror = _HostMirror(copy_device, self.shadow, self.pin_memory) if copy_device is not None else None

    # ---------------------------------------------------------------- attributes kept from the reference
    decay = property(lambda self: self._sched.decay)
    profile = property(lambda self: self._sched.profile)
    gamma = property(lambda self: self._sched.gamma)
    update_every = property(lambda self: self._sched.update_every)
    num_updates = property(lambda self: self._sched.num_updates)

    @staticmethod
    def _tracked(model: torch.nn.Module) -> Iterator[Tuple[str, torch.nn.Parameter]]:
        return ((n, p) for n, p in model.named_parameters() if p.requires_grad)

    def _shadowed(self, model: torch.nn.Module) -> Iterator[Tuple[str, torch.nn.Parameter]]:
        return ((n, p) for n, p in self._tracked(model) if n in self.shadow)

    # ---------------------------------------------------------------- updates
    def fusable(self) -> bool:
        """True when the shadows are fp32 tensors on CUDA (a fused optimizer can update them)."""

        return (not self.offload and self.dtype == torch.float32 and bool(self.shadow)
                and all(t.is_cuda for t in self.shadow.values()))

    def begin_fused_update(self, model: torch.nn.Module, decay: Optional[float] = None
                           ) -> Optional[Tuple[float, Dict[int, torch.Tensor]]]:
        """Hand this step's update to a fused optimizer.

        Returns ``(d, {id(param): shadow})`` when an update is due -- the
        caller then applies ``shadow = d * shadow + (1 - d) * new_param`` to
        every listed parameter -- or None when thinning skips this step.
        """

        d = self._sched.advance(decay)
        if d is None:
            return None
        self._sched.mark_applied()
        return d, {id(p): self.shadow[n] for n, p in self._shadowed(model)}

    def _blend(self, targets: Dict[str, torch.Tensor], d: float) -> None:
        for name, src in targets.items():
            self.shadow[name].mul_(d).add_(src, alpha=1.0 - d)

    @torch.no_grad()
    def update(self, model: torch.nn.Module, decay: Optional[float] = None) -> None:
        d = self._sched.advance(decay)
        if d is None:
            return
        if self._mirror is not None:
            self._mirror.drain()  # the previous snapshot's math is done before its staging is reused
            self._mirror.snapshot(self._shadowed(model), self.dtype, lambda staged: self._blend(staged, d))
            self._sched.mark_applied()
            return
        native_dst: List[torch.Tensor] = []
        native_src: List[torch.Tensor] = []
        by_kind: Dict[Tuple[torch.device, torch.dtype], Tuple[List[torch.Tensor], List[torch.Tensor]]] = {}
        for name, p in self._shadowed(model):
            dst, src = self.shadow[name], p.detach()
            if (dst.is_cuda and src.device == dst.device and dst.dtype == src.dtype == torch.float32
                    and dst.is_contiguous() and src.is_contiguous()):
                native_dst.append(dst)
                native_src.append(src)
            elif dst.dtype in (torch.float32, torch.float64):
                pair = by_kind.setdefault((dst.device, dst.dtype), ([], []))
                pair[0].append(dst)
                pair[1].append(src.to(device=dst.device, dtype=self.dtype))
            else:
                dst.mul_(d).add_(src.to(device=dst.device, dtype=self.dtype), alpha=1.0 - d)
        if native_dst:
            from ..ops._ext import native

            native().ema_update(native_dst, native_src, float(d))
        for dsts, srcs in by_kind.values():
            torch._foreach_mul_(dsts, d)
            torch._foreach_add_(dsts, srcs, alpha=1.0 - d)
        self._sched.mark_applied()

    def wait_before_param_mutation(self) -> None:
        if self._mirror is not None:
            self._mirror.release_params()

    @torch.no_grad()
    def flush(self) -> None:
        if self._mirror is not None:
            self._mirror.drain()

    # ---------------------------------------------------------------- state (checkpoint format)
    def state_dict(self, clone: bool = False) -> Dict[str, object]:
        self.flush()
        s = self._sched
        return {
            "decay": s.decay, "profile": s.profile, "gamma": None if s.gamma is None else float(s.gamma),
            "num_updates": s.num_updates, "step_counter": s.step_counter, "last_update_step_counter": s.last_update,
            "update_every": s.update_every, "compensate_update_every": self.compensate_update_every,
            "shadow": {k: v.clone() if clone else v for k, v in self.shadow.items()}, "dtype": str(self.dtype),
        }

    @torch.no_grad()
    def load_state_dict(self, state: Dict[str, object]) -> None:
        self.flush()
        s = self._sched

        def number(key: str, default):
            value = state.get(key, default)
            return value if isinstance(value, (int, float)) and not isinstance(value, bool) else default

        s.decay = float(number("decay", s.decay))
        if isinstance(state.get("profile"), str):
            s.profile = str(state["profile"]).lower()
        if number("gamma", None) is not None:
            s.gamma = float(state["gamma"])  # type: ignore[arg-type]
        s.num_updates = int(number("num_updates", 0))
        s.step_counter = int(number("step_counter", s.num_updates))
        s.update_every = max(1, int(number("update_every", s.update_every)))
        last = number("last_update_step_counter", None)
        if last is not None:
            s.last_update = max(0, int(last))
        else:  # older checkpoints: the last multiple of update_every
            step = max(0, s.step_counter)
            s.last_update = step - step % s.update_every
        self.compensate_update_every = True
        for name, value in (state.get("shadow") or {}).items():  # type: ignore[union-attr]
            if name in self.shadow and isinstance(value, torch.Tensor):
                self.shadow[name].copy_(value.to(dtype=self.dtype, device=self.shadow[name].device))

    # ---------------------------------------------------------------- evaluation with the averaged weights
    @torch.no_grad()
    def store(self, model: torch.nn.Module) -> None:
        self._saved = {n: p.detach().clone() for n, p in self._tracked(model)}

    @torch.no_grad()
    def copy_to(self, model: torch.nn.Module) -> None:
        self.flush()
        for name, p in self._shadowed(model):
            p.data.copy_(self.shadow[name].to(device=p.device, dtype=p.dtype))

    @torch.no_grad()
    def restore(self, model: torch.nn.Module) -> None:
        if self._saved is None:
            return
        for name, p in self._tracked(model):
            if name in self._saved:
                p.data.copy_(self._saved[name])
        self._saved = None

    # Kept for callers of the reference's class methods.
    _srel_from_gamma = staticmethod(_srel_of_gamma)
    _gamma_from_srel = staticmethod(_gamma_of_srel)
