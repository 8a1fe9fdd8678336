"""Pieces shared by the benchmark models.

* ``compute_dtype()`` reads the active autocast dtype: under bf16/fp16
  autocast on CUDA the models run on the native sm_100a kernels with fp32
  master parameters (the same numerics contract as autocast: fp32 params,
  low-precision GEMM operands, fp32 accumulation); otherwise they run the
  plain-PyTorch reference path.
* ``LowPrecisionShadows`` keeps a bf16/fp16 copy of every GEMM weight. A copy
  is refreshed only when its parameter changed through PyTorch (tracked by the
  tensor version counter); the fused optimizer writes the copies itself in the
  same pass that updates the parameters.
"""

from __future__ import annotations

from typing import Dict, Iterable, List, Optional

import torch
import torch.nn as nn

from ..ops import functional as kf


def compute_dtype(device: torch.device) -> Optional[torch.dtype]:
    """Low-precision compute dtype for native kernels, or None for the reference path."""

    if device.type != "cuda":
        return None
    if not torch.is_autocast_enabled("cuda"):
        return None
    dt = torch.get_autocast_dtype("cuda")
    return dt if dt in (torch.bfloat16, torch.float16) else None


def shadow_of(param: torch.Tensor, dtype: torch.dtype) -> Optional[torch.Tensor]:
    sh = getattr(param, "_kb_shadow", None)
    if sh is None or sh.dtype != dtype or sh.device != param.device or sh.shape != param.shape:
        return None
    return sh


class LowPrecisionShadows:
    """bf16/fp16 copies of a fixed list of fp32 matrix parameters."""

    def __init__(self, params: Iterable[nn.Parameter]) -> None:
        self.params: List[nn.Parameter] = list(params)

    def get(self, dtype: torch.dtype) -> Dict[int, torch.Tensor]:
        stale_src: List[torch.Tensor] = []
        stale_dst: List[torch.Tensor] = []
        out: Dict[int, torch.Tensor] = {}
        for p in self.params:
            sh = shadow_of(p, dtype)
            if sh is None:
                sh = torch.empty(p.shape, device=p.device, dtype=dtype)
                p._kb_shadow = sh  # type: ignore[attr-defined]
                p._kb_shadow_version = -1  # type: ignore[attr-defined]
            if getattr(p, "_kb_shadow_version", -1) != p._version:
                stale_src.append(p.detach())
                stale_dst.append(sh)
                p._kb_shadow_version = p._version  # type: ignore[attr-defined]
            out[id(p)] = sh
        if stale_src:
            kf.cast_multi(stale_src, stale_dst)
        return out


def mark_shadow_fresh(param: torch.Tensor) -> None:
    """Called by kernels that rewrote ``param`` and its shadow together."""

    if getattr(param, "_kb_shadow", None) is not None:
        param._kb_shadow_version = param._version  # type: ignore[attr-defined]


def to_lp(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp32 -> bf16/fp16 cast on the native kernel (contiguous input)."""

    t = t.contiguous()
    out = torch.empty(t.shape, device=t.device, dtype=dtype)
    kf.cast_multi([t], [out])
    return out
