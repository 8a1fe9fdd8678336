"""Joint-L2 gradient clipping that never squares huge values in their own scale.

(reference: koochak/optim/grad_clip.py:11-73)

``clip_grad_norm_`` (PyTorch ops, one device-to-host read) is the reference
behaviour. ``fused_grad_gate`` is the native equivalent used by the training
loop on CUDA: one multi-tensor pass computes per-tensor sums of squares and a
non-finite flag (and, for fp16, unscales in place), a one-thread kernel forms
the global norm (fp64 combine of per-tensor fp32 norms) and the coefficient
``min(1, max_norm / (norm + 1e-6))`` on the device, and the host reads the
three numbers once. The coefficient is not written back into the gradients:
the fused optimizers read gradients through it. When the plain norm
overflows fp32 while every entry is finite, the overflow-safe scaled path of
``clip_grad_norm_`` runs instead, so results match the reference.
"""

from __future__ import annotations

import math
from typing import Iterable, List, NamedTuple, Optional, Sequence

import torch

__all__ = ["GradientClipStats", "clip_grad_norm_", "fused_grad_gate", "GateResult"]


class GradientClipStats(NamedTuple):
    norm: float
    coefficient: float
    used_scaled_norm: bool


def _global_norm(norms: Iterable[torch.Tensor]) -> float:
    values = torch.stack(tuple(norms))
    if values.device.type == "mps":
        values = values.cpu()
    return float(values.double().norm())


def _scaled_norm(grad: torch.Tensor, root: float) -> torch.Tensor:
    scaled = grad / root
    scaled.div_(root)
    return scaled.norm()


def _scaled_clip(grads: List[torch.Tensor], maximum: float) -> GradientClipStats:
    largest = float(torch.stack(torch._foreach_norm(grads, math.inf)).max())
    if not math.isfinite(largest):
        raise FloatingPointError("Gradient entries contain NaN or infinity; optimizer step stopped.")
    root = math.sqrt(largest)  # two normal-range factors avoid a subnormal reciprocal
    scaled = _global_norm(_scaled_norm(g, root) for g in grads)
    norm = largest * scaled
    coef = min(1.0, (maximum / largest) / (scaled + 1e-6 / largest))
    if coef < 1.0:
        half = math.sqrt(coef)
        torch._foreach_mul_(grads, half)
        torch._foreach_mul_(grads, half)
    return GradientClipStats(norm, coef, True)


def _dense_grads(parameters) -> List[torch.Tensor]:
    grads = [p.grad.detach() for p in parameters if p.grad is not None and p.grad.numel()]
    if any(g.layout != torch.strided or not g.is_floating_point() for g in grads):
        raise TypeError("Gradient clipping requires dense floating-point gradients.")
    if grads and any(g.device != grads[0].device for g in grads):
        raise ValueError("Gradient clipping requires all gradients on the same device.")
    return grads


@torch.no_grad()
def clip_grad_norm_(parameters: Iterable[torch.Tensor], max_norm: float) -> GradientClipStats:
    """Clip the joint L2 norm in place; raise FloatingPointError on non-finite entries."""

    maximum = float(max_norm)
    if not math.isfinite(maximum) or maximum < 0.0:
        raise ValueError("max_norm must be finite and nonnegative.")
    grads = _dense_grads(parameters)
    if not grads:
        return GradientClipStats(0.0, 1.0, False)
    norm = _global_norm(torch._foreach_norm(grads, 2.0))
    coef = min(1.0, maximum / (norm + 1e-6))
    tiny = 0.0 < coef < torch.finfo(torch.float32).tiny
    if not math.isfinite(norm) or tiny:
        return _scaled_clip(grads, maximum)
    torch._foreach_mul_(grads, coef)
    return GradientClipStats(norm, coef, False)


class GateResult(NamedTuple):
    stats: Optional[GradientClipStats]   # None when clipping is off
    coef_tensor: Optional[torch.Tensor]  # device scalar to apply on read (None: nothing to apply)
    nonfinite: bool
    device_stats: Optional[torch.Tensor] = None  # fp32 [norm, coefficient, found_inf] on the device


@torch.no_grad()
def fused_grad_gate(grads: Sequence[torch.Tensor], *, max_norm: Optional[float], check_finite: bool,
                    inv_scale: Optional[torch.Tensor] = None, sync: bool = True) -> GateResult:
    """One native pass over CUDA fp32 gradients: unscale?, finite flag, norm, clip coefficient."""

    from ..ops._ext import native

    clip = max_norm is not None
    if clip:
        maximum = float(max_norm)
        if not math.isfinite(maximum) or maximum < 0.0:
            raise ValueError("max_norm must be finite and nonnegative.")
    grads = [g for g in grads if g.numel()]
    if not grads:
        return GateResult(GradientClipStats(0.0, 1.0, False) if clip else None, None, False)
    dev = grads[0].device
    scratch = torch.empty(len(grads) + 1, device=dev, dtype=torch.float64)
    out = torch.empty(3, device=dev, dtype=torch.float32)
    native().grad_stats(list(grads), inv_scale, float(max_norm or 0.0), clip, scratch, out, None)
    coef_t = out[1:2]
    if not (clip or check_finite) or not sync:
        return GateResult(None, coef_t if clip else None, False, out)
    norm, coef, bad = (float(v) for v in out.tolist())
    nonfinite = bad != 0.0
    if not clip:
        return GateResult(None, None, nonfinite)
    if nonfinite or not math.isfinite(norm) or (0.0 < coef < torch.finfo(torch.float32).tiny):
        finite = all(bool(torch.isfinite(g).all()) for g in grads)
        if not finite:
            raise FloatingPointError("Gradient entries contain NaN or infinity; optimizer step stopped.")
        stats = _scaled_clip(list(grads), float(max_norm))  # overflow-safe path, writes grads
        return GateResult(stats, None, False)
    return GateResult(GradientClipStats(norm, coef, False), coef_t, False)
