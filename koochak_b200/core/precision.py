"""Autocast contexts and the gradient scaler (reference: koochak/core/precision.py:18-85).

``Scaler("fp16")`` on CUDA returns :class:`FusedGradScaler`, a
``torch.amp.GradScaler`` whose ``unscale_`` runs one native pass over all
gradients: unscale in place, non-finite detection, and (for the training
loop's gradient gate) the per-tensor squared norms used by clipping. Its
``state_dict`` is the stock GradScaler one, so checkpoints stay compatible.
Any other mode returns a no-op scaler with the same interface.
"""

from __future__ import annotations

from contextlib import nullcontext
from typing import Any, Dict, List, Optional

import torch
from torch.amp import GradScaler, autocast

__all__ = ["autocast_context", "Scaler", "is_fp16", "prepare_compile_backend", "FusedGradScaler", "NoOpScaler"]

_TF32_PATCH_ATTR = "__koochak_tf32_state_key_patch__"


def is_fp16(mode: Optional[str]) -> bool:
    return (mode or "fp32").lower() == "fp16"


def autocast_context(mode: Optional[str], device: torch.device):
    mode = (mode or "fp32").lower()
    if mode == "fp16":
        return autocast(device_type="cuda" if device.type == "cuda" else "cpu", dtype=torch.float16)
    if mode == "bf16":
        return autocast(device_type=device.type, dtype=torch.bfloat16)
    return nullcontext()


def _tf32_enabled_by_precision() -> bool:
    if not hasattr(torch.backends.cuda.matmul, "fp32_precision"):
        return bool(torch._C._get_cublas_allow_tf32())
    return str(torch.backends.cuda.matmul.fp32_precision).strip().lower() != "ieee"


def prepare_compile_backend() -> None:
    """Make Dynamo's global-state key read TF32 through the new precision API.

    Without this, torch versions that expose ``fp32_precision`` can warn or
    recompile when the legacy TF32 getter is queried.
    """

    if not hasattr(torch.backends.cuda.matmul, "fp32_precision"):
        return
    try:
        from torch._dynamo import graph_region_tracker
    except ImportError:
        return
    current = getattr(graph_region_tracker, "get_global_state_key", None)
    if current is None or getattr(current, _TF32_PATCH_ATTR, False):
        return

    def _key():
        return (
            torch.is_grad_enabled(),
            torch.is_inference_mode_enabled(),
            torch.get_num_threads(),
            torch._C._get_cublas_allow_fp16_reduced_precision_reduction(),
            torch._C._get_cublas_allow_bf16_reduced_precision_reduction(),
            torch.get_default_dtype(),
            torch.are_deterministic_algorithms_enabled(),
            _tf32_enabled_by_precision(),
            torch.is_deterministic_algorithms_warn_only_enabled(),
            torch._C._autograd._saved_tensors_hooks_is_enabled(),  # type: ignore[attr-defined]
        )

    setattr(_key, _TF32_PATCH_ATTR, True)
    graph_region_tracker.get_global_state_key = _key


class NoOpScaler:
    """Scaler interface for fp32/bf16 runs: every call passes through."""

    def scale(self, loss):
        return loss

    def step(self, optimizer):
        optimizer.step()

    def update(self):
        pass

    def unscale_(self, optimizer):
        pass

    def state_dict(self):
        return {}


_NoOpScaler = NoOpScaler  # name used by older callers


def _grads_of(optimizer) -> List[torch.Tensor]:
    out = []
    for group in optimizer.param_groups:
        for p in group["params"]:
            if p.grad is not None:
                out.append(p.grad)
    return out


class FusedGradScaler(GradScaler):
    """GradScaler whose unscale/finite-check is one native multi-tensor pass."""

    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        self.last_stats: Optional[torch.Tensor] = None

    def unscale_(self, optimizer, *, max_norm: Optional[float] = None) -> None:  # type: ignore[override]
        from torch.amp.grad_scaler import OptState

        self.last_stats = None
        if not self._enabled:
            return
        self._check_scale_growth_tracker("unscale_")
        state = self._per_optimizer_states[id(optimizer)]
        if state["stage"] is OptState.UNSCALED:
            raise RuntimeError("unscale_() has already been called on this optimizer since the last update().")
        if state["stage"] is OptState.STEPPED:
            raise RuntimeError("unscale_() is being called after step().")
        grads = _grads_of(optimizer)
        native_ok = bool(grads) and all(
            g.is_cuda and g.dtype == torch.float32 and g.is_contiguous() and not g.is_sparse for g in grads)
        if not native_ok:
            super().unscale_(optimizer)
            return
        from ..ops._ext import native

        assert self._scale is not None
        inv_scale = self._scale.double().reciprocal().float()
        dev = grads[0].device
        scratch = torch.empty(len(grads) + 1, device=dev, dtype=torch.float64)
        stats = torch.empty(3, device=dev, dtype=torch.float32)
        native().grad_stats(grads, inv_scale, float(max_norm or 0.0), max_norm is not None, scratch, stats, None)
        found_inf = stats[2:3].clone()
        state["found_inf_per_device"] = {dev: found_inf}
        state["stage"] = OptState.UNSCALED
        self.last_stats = stats


    def mark_unscaled(self, optimizer, stats: torch.Tensor) -> None:
        """Record gradients that were already unscaled elsewhere (the fused all-reduce).

        ``stats`` is the device vector [norm, coefficient, found_inf, ...] of
        that pass; its found_inf decides whether ``step`` is skipped.
        """

        from torch.amp.grad_scaler import OptState

        if not self._enabled:
            return
        self._check_scale_growth_tracker("unscale_")
        state = self._per_optimizer_states[id(optimizer)]
        if state["stage"] is not OptState.READY:
            raise RuntimeError("mark_unscaled() must come before unscale_() / step() of this update.")
        dev = stats.device
        state["found_inf_per_device"] = {dev: stats[2:3].clone()}
        state["stage"] = OptState.UNSCALED
        self.last_stats = stats


def Scaler(mode: Optional[str]):
    """GradScaler for fp16 on CUDA, a no-op scaler otherwise."""

    if is_fp16(mode) and torch.cuda.is_available():
        return FusedGradScaler(enabled=True)
    return NoOpScaler()
