"""Exponential moving average of trainable parameters (reference: koochak/utils/ema.py:6-327).

Shadows are fp32 copies keyed by parameter name (the checkpoint format).

* GPU-resident shadows (``offload_to_cpu=False``) are updated with one native
  multi-tensor kernel; when the optimizer is a fused one from this package,
  the update is folded into the optimizer's own parameter-update pass
  (``begin_fused_update`` hands it the decay for this step).
* CPU-offloaded shadows (the default, as in the reference) copy a snapshot of
  the parameters device-to-host on a side stream after each update and apply
  the math on a single background thread; ``wait_before_param_mutation``
  blocks until that snapshot no longer reads live parameters.

Decay: ``profile="constant"`` uses d (compensated to d**N when updates are
thinned to every N steps); ``profile="power"`` uses ((t-N)/t)^(gamma+1).
"""

from __future__ import annotations

import math
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Dict, List, Optional, Tuple

import torch

__all__ = ["EMA"]


class EMA:
    def __init__(self, model: torch.nn.Module, decay: float = 0.999, *, dtype: torch.dtype = torch.float32,
                 profile: str = "constant", gamma: Optional[float] = None, srel: Optional[float] = None,
                 update_every: int = 1, offload_to_cpu: bool = True, pin_memory: bool = True,
                 compensate_update_every: bool = True) -> None:
        if not 0.0 < float(decay) < 1.0:
            raise ValueError("EMA decay must be in (0, 1)")
        self.decay = float(decay)
        self.dtype = dtype
        self.offload = bool(offload_to_cpu)
        self.pin_memory = bool(pin_memory)
        self.update_every = max(1, int(update_every))
        # Thinned updates are always compensated; the flag is kept for the checkpoint format.
        self.compensate_update_every = True
        self.profile = (profile or "constant").lower()
        if self.profile not in ("constant", "power"):
            raise ValueError(f"Unsupported EMA profile: {self.profile}")
        self.gamma = float(gamma) if gamma is not None else (self._gamma_from_srel(float(srel)) if srel is not None
                                                             else None)
        self.shadow: Dict[str, torch.Tensor] = {}
        self.staging: Dict[str, torch.Tensor] = {}
        self.pending_event: Dict[str, Optional["torch.cuda.Event"]] = {}
        self.pending_decay: Dict[str, float] = {}
        self._copy_device: Optional[torch.device] = None
        self._copy_stream: Optional["torch.cuda.Stream"] = None
        self._copy_done: Optional["torch.cuda.Event"] = None
        self._worker: Optional[ThreadPoolExecutor] = None
        self._worker_future: Optional[Future] = None
        self.num_updates = 0
        self._step_counter = 0
        self._last_update_step_counter = 0
        self._backup: Optional[Dict[str, torch.Tensor]] = None
        self._build(model)

    # ------------------------------------------------------------ decay math
    @staticmethod
    def _srel_from_gamma(gamma: float) -> float:
        g = float(gamma)
        return math.sqrt(g + 1.0) / ((g + 2.0) * math.sqrt(g + 3.0))

    @classmethod
    def _gamma_from_srel(cls, srel: float) -> float:
        target = max(1e-9, float(srel))
        lo, hi = 1e-6, 1e6
        for _ in range(64):
            mid = math.sqrt(lo * hi)
            if cls._srel_from_gamma(mid) > target:
                lo = mid
            else:
                hi = mid
        return 0.5 * (lo + hi)

    def _current_decay(self, elapsed_steps: int = 1) -> float:
        if self.profile == "constant":
            return float(self.decay)
        g = float(self.gamma if self.gamma is not None else 6.94)
        t = max(1.0, float(self._step_counter))
        prev = max(0.0, t - float(max(1, int(elapsed_steps))))
        return float((prev / t) ** (g + 1.0))

    def _effective_decay(self, decay: Optional[float], elapsed_steps: int) -> float:
        d = float(self._current_decay(elapsed_steps) if decay is None else decay)
        if self.profile == "constant":
            d = d ** float(max(1, int(elapsed_steps)))
        return d

    # ------------------------------------------------------------ construction
    def _build(self, model: torch.nn.Module) -> None:
        for name, p in model.named_parameters():
            if not p.requires_grad:
                continue
            dev = torch.device("cpu") if self.offload else p.device
            self.shadow[name] = p.detach().to(device=dev, dtype=self.dtype).clone()
            if self.offload:
                self.staging[name] = torch.empty_like(self.shadow[name], device="cpu",
                                                      pin_memory=p.is_cuda and self.pin_memory)
            self.pending_event[name] = None
            self.pending_decay[name] = self.decay
            if self.offload and p.is_cuda and self._copy_device is None:
                self._copy_device = p.device
        if self._copy_device is not None:
            with torch.cuda.device(self._copy_device):
                self._copy_stream = torch.cuda.Stream(device=self._copy_device)
            self._worker = ThreadPoolExecutor(max_workers=1, thread_name_prefix="koochak-ema")

    # ------------------------------------------------------------ updates
    def _advance(self, decay: Optional[float]) -> Optional[float]:
        """Step the counters; the decay to apply now, or None when thinned out."""

        self._step_counter += 1
        if self.update_every > 1 and self._step_counter % self.update_every != 0:
            return None
        elapsed = max(1, int(self._step_counter - self._last_update_step_counter))
        d = self._effective_decay(decay, elapsed)
        self.num_updates += 1
        return d

    def fusable(self) -> bool:
        """True when shadows are fp32 tensors on the parameters' CUDA device."""

        return (not self.offload and self.dtype == torch.float32 and bool(self.shadow)
                and all(s.is_cuda for s in self.shadow.values()))

    def begin_fused_update(self, model: torch.nn.Module, decay: Optional[float] = None
                           ) -> Optional[Tuple[float, Dict[int, torch.Tensor]]]:
        """Reserve this step's update for a fused optimizer.

        Returns ``(d, {id(param): shadow})`` when an update is due (the caller
        must then apply ``shadow = d*shadow + (1-d)*param_new`` to every listed
        parameter), or None when thinning skips this step.
        """

        d = self._advance(decay)
        if d is None:
            return None
        self._last_update_step_counter = self._step_counter
        by_id = {}
        for name, p in model.named_parameters():
            if p.requires_grad and name in self.shadow:
                by_id[id(p)] = self.shadow[name]
        return d, by_id

    @torch.no_grad()
    def update(self, model: torch.nn.Module, decay: Optional[float] = None) -> None:
        d = self._advance(decay)
        if d is None:
            return
        self._wait_worker()
        if self._copy_stream is not None and self._copy_device is not None:
            self._snapshot_async(model, d)
            self._last_update_step_counter = self._step_counter
            return
        cuda_dst: List[torch.Tensor] = []
        cuda_src: List[torch.Tensor] = []
        groups: Dict[Tuple[torch.device, torch.dtype], Tuple[List[torch.Tensor], List[torch.Tensor]]] = {}
        for name, p in model.named_parameters():
            if not p.requires_grad or name not in self.shadow:
                continue
            dst = self.shadow[name]
            src = p.detach()
            if (dst.is_cuda and dst.dtype == torch.float32 and src.dtype == torch.float32 and src.device == dst.device
                    and src.is_contiguous() and dst.is_contiguous()):
                cuda_dst.append(dst)
                cuda_src.append(src)
                continue
            src = src.to(device=dst.device, dtype=self.dtype)
            if dst.dtype not in (torch.float32, torch.float64):
                dst.mul_(d).add_(src, alpha=1.0 - d)
                continue
            ds, ss = groups.setdefault((dst.device, dst.dtype), ([], []))
            ds.append(dst)
            ss.append(src)
        if cuda_dst:
            from ..ops._ext import native

            native().ema_update(cuda_dst, cuda_src, float(d))
        for ds, ss in groups.values():
            torch._foreach_mul_(ds, d)
            torch._foreach_add_(ds, ss, alpha=1.0 - d)
        self._last_update_step_counter = self._step_counter

    def wait_before_param_mutation(self) -> None:
        ev = self._copy_done
        if ev is None:
            return
        if not torch.cuda.is_available():
            raise RuntimeError("EMA has a pending CUDA snapshot but CUDA is not available on this process")
        ev.synchronize()
        self._copy_done = None

    # ------------------------------------------------------------ state
    def state_dict(self, clone: bool = False) -> Dict[str, object]:
        self.flush()
        return {
            "decay": self.decay, "profile": self.profile,
            "gamma": float(self.gamma) if self.gamma is not None else None,
            "num_updates": self.num_updates, "step_counter": self._step_counter,
            "last_update_step_counter": self._last_update_step_counter, "update_every": self.update_every,
            "compensate_update_every": self.compensate_update_every,
            "shadow": {k: (v.clone() if clone else v) for k, v in self.shadow.items()},
            "dtype": str(self.dtype),
        }

    @torch.no_grad()
    def load_state_dict(self, state: Dict[str, object]) -> None:
        self.flush()
        if isinstance(state.get("decay", self.decay), (int, float)):
            self.decay = float(state.get("decay", self.decay))  # type: ignore[arg-type]
        if isinstance(state.get("profile", self.profile), str):
            self.profile = str(state.get("profile", self.profile)).lower()
        if isinstance(state.get("gamma"), (int, float)):
            self.gamma = float(state["gamma"])  # type: ignore[arg-type]
        nu = state.get("num_updates", 0)
        self.num_updates = int(nu) if isinstance(nu, (int, float)) else 0
        sc = state.get("step_counter", self.num_updates)
        self._step_counter = int(sc) if isinstance(sc, (int, float)) else self.num_updates
        ue = state.get("update_every", self.update_every)
        if isinstance(ue, (int, float)):
            self.update_every = max(1, int(ue))
        last = state.get("last_update_step_counter")
        if isinstance(last, (int, float)):
            self._last_update_step_counter = max(0, int(last))
        else:
            step, every = max(0, self._step_counter), max(1, self.update_every)
            self._last_update_step_counter = step if every == 1 else step - step % every
        self.compensate_update_every = True
        shadow = state.get("shadow", {})
        if isinstance(shadow, dict):
            for k, v in shadow.items():
                if k in self.shadow and isinstance(v, torch.Tensor):
                    dst = self.shadow[k]
                    dst.copy_(v.to(dtype=self.dtype, device=dst.device))

    # ------------------------------------------------------------ eval helpers
    @torch.no_grad()
    def store(self, model: torch.nn.Module) -> None:
        self._backup = {n: p.detach().clone() for n, p in model.named_parameters() if p.requires_grad}

    @torch.no_grad()
    def copy_to(self, model: torch.nn.Module) -> None:
        self.flush()
        for n, p in model.named_parameters():
            if p.requires_grad and n in self.shadow:
                p.data.copy_(self.shadow[n].to(device=p.device, dtype=p.dtype))

    @torch.no_grad()
    def restore(self, model: torch.nn.Module) -> None:
        if self._backup is None:
            return
        for n, p in model.named_parameters():
            if p.requires_grad and n in self._backup:
                p.data.copy_(self._backup[n])
        self._backup = None

    # ------------------------------------------------------------ offload internals
    def _wait_worker(self) -> None:
        fut = self._worker_future
        if fut is not None:
            fut.result()
            self._worker_future = None

    @torch.no_grad()
    def _apply_staged(self, decay: float) -> None:
        for name, dst in self.shadow.items():
            dst.mul_(decay).add_(self.staging[name], alpha=1.0 - decay)

    @torch.no_grad()
    def _apply_after(self, event: "torch.cuda.Event", decay: float) -> None:
        event.synchronize()
        self._apply_staged(decay)

    @torch.no_grad()
    def _apply_ready_staged(self) -> None:
        if self._copy_done is not None:
            if not self._copy_done.query():
                return
            self._copy_done = None
        for name, ev in self.pending_event.items():
            if ev is None or not ev.query():
                continue
            d = self.pending_decay.get(name, self.decay)
            self.shadow[name].mul_(d).add_(self.staging[name], alpha=1.0 - d)
            self.pending_event[name] = None

    @torch.no_grad()
    def _snapshot_async(self, model: torch.nn.Module, decay: float) -> None:
        assert self._copy_device is not None and self._copy_stream is not None and self._worker is not None
        with torch.cuda.device(self._copy_device):
            ready = torch.cuda.Event(blocking=False)
            done = torch.cuda.Event(blocking=False)
            ready.record(torch.cuda.current_stream(self._copy_device))
            with torch.cuda.stream(self._copy_stream):
                self._copy_stream.wait_event(ready)
                for name, p in model.named_parameters():
                    if not p.requires_grad or name not in self.shadow:
                        continue
                    src = p.detach()
                    if src.dtype is not self.dtype:
                        src = src.to(dtype=self.dtype)
                    self.staging[name].copy_(src, non_blocking=True)
                    self.pending_decay[name] = decay
                done.record(self._copy_stream)
        self._copy_done = done
        self._worker_future = self._worker.submit(self._apply_after, done, decay)

    @torch.no_grad()
    def flush(self) -> None:
        self.wait_before_param_mutation()
        self._wait_worker()
        for name in self.pending_event:
            self.pending_event[name] = None
