"""The gradient gate between backward and the optimizer: unscale, finite check, clip.

(semantics of reference koochak/loop.py:1612-1637 and koochak/optim/grad_clip.py)

The order and the outcome are the reference's: unscale fp16 gradients, run
the periodic non-finite check (``FloatingPointError`` naming the tensors),
then clip to ``grad_clip_norm`` (the joint L2 norm, combined in fp64;
``FloatingPointError`` when it is not finite). Where the numbers come from
depends on the run, most direct source first:

1. the fused data-parallel sync already averaged, unscaled and measured the
   gradients: one seal kernel and one 16-byte read (``DataParallel.fused_gate``);
2. single process on CUDA with the native scaler: one native pass over the
   gradients (``FusedGradScaler.unscale_``);
3. CUDA fp32 gradients: ``fused_grad_gate`` (one native pass, no unscale);
4. anything else: torch's unscale and the reference-style clip.

A fused optimizer from this package takes the clip coefficient as a device
scalar and applies it when it reads each gradient (``kb_grad_scale``); other
optimizers get their gradients multiplied in place.
"""

from __future__ import annotations

import math
from typing import Any, Callable, Dict, List, Optional

import torch
from torch.amp import GradScaler

from ..core.precision import FusedGradScaler
from ..optim.grad_clip import GradientClipStats, clip_grad_norm_, fused_grad_gate

__all__ = ["GradientGate", "nonfinite_parameter_names"]


def nonfinite_parameter_names(model: torch.nn.Module) -> List[str]:
    return [name for name, p in model.named_parameters()
            if p.grad is not None and torch.is_floating_point(p.grad) and not bool(torch.isfinite(p.grad).all())]


def _takes_device_coefficient(optimizer: Any) -> bool:
    return any(bool(getattr(o, "kb_fused", False)) for o in (optimizer, getattr(optimizer, "inner", None)))


def _device_coefficient_target(optimizer: Any) -> Any:
    """The fused optimizer (this one or the one a wrapper holds) that takes device coefficient and skip flag."""

    for o in (optimizer, getattr(optimizer, "inner", None)):
        if bool(getattr(o, "kb_fused", False)):
            return o
    return None


class _Pending:
    """A gate result still on the device: its copy to host memory and the event that marks it complete."""

    def __init__(self, stats: torch.Tensor, clip: bool) -> None:
        self.host = torch.empty(stats.numel(), dtype=torch.float32, pin_memory=True)
        self.host.copy_(stats, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record()
        self.clip = clip

    def values(self) -> List[float]:
        self.event.synchronize()
        return [float(v) for v in self.host.tolist()]


class GradientGate:
    """Unscale, finite check and clip between backward and the optimizer, in two phases.

    ``begin`` computes the gate on the device. When the optimizer is one of
    this package's fused optimizers, it hands the clip coefficient and the
    found-inf flag over as device scalars (``kb_grad_scale``, ``kb_skip``)
    and starts a non-blocking copy of the statistics to host memory, so the
    optimizer step is enqueued without waiting for the gate's result; the
    optimizer kernels skip the update on the device when the flag is set.
    ``finish`` (after the optimizer step was enqueued, before anything that
    depends on its outcome) reads the statistics -- by then the GPU is busy
    with the optimizer kernels, so the wait costs it nothing -- and applies
    the reference's outcome: a rejected step under clipping raises
    ``FloatingPointError`` (the update was skipped on the device and the
    optimizer rolls back its host-side step counters, so the state is the
    one the reference leaves), a rejected step without clipping is the
    GradScaler skip. Other optimizers get the synchronous gate in ``begin``.
    """

    def __init__(self, *, max_norm: Optional[float], check_every: int, scaler: Any,
                 profile: Callable[[str, Callable[[], Any]], Any]) -> None:
        self.max_norm = None if max_norm is None else float(max_norm)
        self.check_every = int(check_every)
        self.scaler = scaler
        self.profile = profile  # profile(phase_key, thunk) runs thunk under the loop's step profiler
        self._pending: Optional[_Pending] = None
        self._result: Dict[str, Any] = {}
        self._owner: Any = None

    @staticmethod
    def _native_gradients(model: torch.nn.Module, on_cuda: bool) -> Optional[List[torch.Tensor]]:
        """Every gradient, if all are dense fp32 CUDA tensors and the native library is loaded."""

        if not on_cuda:
            return None
        grads = [p.grad for p in model.parameters() if p.grad is not None]
        plain = all(g.is_cuda and g.dtype == torch.float32 and g.is_contiguous() and g.layout == torch.strided
                    for g in grads)
        if not grads or not plain:
            return None
        from ..ops._ext import available

        return grads if available() else None

    def run(self, model: torch.nn.Module, optimizer: Any, step: int, on_cuda: bool) -> Dict[str, Any]:
        """Both phases at once, for callers that step the optimizer themselves afterwards."""

        self.begin(model, optimizer, step, on_cuda, defer=False)
        return self.finish(model, optimizer)

    def begin(self, model: torch.nn.Module, optimizer: Any, step: int, on_cuda: bool, defer: bool = True) -> None:
        self._pending, self._result, self._owner = None, {}, None
        grads = self._native_gradients(model, on_cuda)
        stats = self.profile("profile_loop_unscale_time_s", lambda: self._unscale(model, optimizer, grads))
        self.profile("profile_loop_nonfinite_grad_check_time_s", lambda: self._check_finite(model, step))
        target = _device_coefficient_target(optimizer)
        if defer and grads is not None and target is not None:
            if stats is None and self.max_norm is not None:
                stats = fused_grad_gate(grads, max_norm=self.max_norm, check_finite=True, sync=False).device_stats
            if stats is not None:
                if self.max_norm is not None:
                    optimizer.kb_grad_scale = stats[1:2]
                optimizer.kb_skip = stats[2:3]
                self._pending = _Pending(stats, self.max_norm is not None)
                self._owner = target
                return
        if self.max_norm is None:
            return
        clip = self.profile("profile_loop_grad_clip_time_s", lambda: self._clip(model, optimizer, grads, stats))
        if isinstance(clip, GradientClipStats):
            self._result = {"grad_norm": clip.norm, "grad_clip_coefficient": clip.coefficient,
                            "grad_clip_scaled_norm": int(clip.used_scaled_norm)}

    def finish(self, model: torch.nn.Module, optimizer: Any) -> Dict[str, Any]:
        """The clip statistics to log; raises where the reference's gate raises (see the class note)."""

        pending, self._pending = self._pending, None
        if pending is None:
            return self._result
        return self.profile("profile_loop_grad_clip_time_s", lambda: self._settle(model, optimizer, pending))

    def _settle(self, model, optimizer, pending: _Pending) -> Dict[str, Any]:
        values = pending.values()  # [norm, coef, found_inf] (+ device status from the fused all-reduce)
        norm, coef, found_inf = values[:3]
        status = values[3] if len(values) > 3 else 0.0
        if status != 0.0:
            from ..ops._ext import check_status

            check_status(torch.device("cuda", torch.cuda.current_device()))
            raise RuntimeError(f"gradient all-reduce reported device status {int(status)}")
        if found_inf or not math.isfinite(norm):
            rollback = getattr(self._owner, "kb_rollback_step", None)
            if callable(rollback):
                rollback()  # the kernels skipped the update; undo the host-side step counters
            if pending.clip:
                # Reference order: the clip sees the non-finite gradients and raises.
                clip = clip_grad_norm_(model.parameters(), self.max_norm)  # type: ignore[arg-type]
                if isinstance(clip, GradientClipStats):
                    return {"grad_norm": clip.norm, "grad_clip_coefficient": clip.coefficient,
                            "grad_clip_scaled_norm": int(clip.used_scaled_norm)}
            return {}
        if not pending.clip:
            return {}
        return {"grad_norm": norm, "grad_clip_coefficient": coef, "grad_clip_scaled_norm": 0}

    def _unscale(self, model, optimizer, grads) -> Optional[torch.Tensor]:
        fused_dp = getattr(model, "fused_gate_available", None)
        if grads is not None and callable(fused_dp) and fused_dp():
            stats = model.fused_gate(self.max_norm)
            if isinstance(self.scaler, FusedGradScaler):
                self.scaler.mark_unscaled(optimizer, stats)
            return stats
        if isinstance(self.scaler, FusedGradScaler) and grads is not None:
            self.scaler.unscale_(optimizer, max_norm=self.max_norm)
            return self.scaler.last_stats
        if isinstance(self.scaler, GradScaler):
            self.scaler.unscale_(optimizer)
        return None

    def _check_finite(self, model, step: int) -> None:
        if self.check_every > 0 and step % self.check_every == 0:
            bad = nonfinite_parameter_names(model)
            if bad:
                raise FloatingPointError("Gradient entries contain NaN or infinity; optimizer step stopped: "
                                         + ", ".join(bad))

    def _apply(self, optimizer, coef: torch.Tensor, grads: List[torch.Tensor]) -> None:
        if _takes_device_coefficient(optimizer):
            optimizer.kb_grad_scale = coef
        else:
            torch._foreach_mul_(grads, coef)

    def _clip(self, model, optimizer, grads, stats: Optional[torch.Tensor]):
        assert self.max_norm is not None
        if grads is None:
            return clip_grad_norm_(model.parameters(), self.max_norm)
        if stats is None:
            res = fused_grad_gate(grads, max_norm=self.max_norm, check_finite=True)
            if res.coef_tensor is not None:
                self._apply(optimizer, res.coef_tensor, grads)
            return res.stats
        values = [float(v) for v in stats.tolist()]  # [norm, coef, found_inf] (+ device status from the sync)
        norm, coef, found_inf = values[:3]
        status = values[3] if len(values) > 3 else 0.0
        if status != 0.0:
            from ..ops._ext import check_status

            check_status(int(stats.device.index or 0))
            raise RuntimeError(f"gradient all-reduce reported device status {int(status)}")
        if found_inf or not math.isfinite(norm) or 0.0 < coef < torch.finfo(torch.float32).tiny:
            # Overflow or huge values: the reference-style clip decides (and raises on inf / nan).
            return clip_grad_norm_(model.parameters(), self.max_norm)
        self._apply(optimizer, stats[1:2], grads)
        return GradientClipStats(norm, coef, False)
