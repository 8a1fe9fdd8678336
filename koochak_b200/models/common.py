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
    """bf16/fp16 copies of a fixed list of fp32 matrix parameters.

    ``fused_groups`` lists groups of matrices with equal column counts whose
    copies should be row blocks of one buffer (for example q, k and v): the
    forward pass then runs one GEMM on the stacked weight while every matrix
    stays its own parameter (Muon orthogonalises each separately).
    """

    def __init__(self, params: Iterable[nn.Parameter], fused_groups: Iterable[Iterable[nn.Parameter]] = ()) -> None:
        self.params: List[nn.Parameter] = list(params)
        self.fused_groups: List[List[nn.Parameter]] = [list(g) for g in fused_groups]
        known = {id(p) for p in self.params}
        for g in self.fused_groups:
            if any(id(p) not in known for p in g) or len({p.shape[1] for p in g}) != 1:
                raise ValueError("fused shadow groups must be listed parameters with equal column counts")
        self._fused: Dict[tuple, torch.Tensor] = {}

    def _ensure_fused(self, dtype: torch.dtype) -> None:
        for gi, g in enumerate(self.fused_groups):
            buf = self._fused.get((gi, dtype))
            if buf is not None and buf.device == g[0].device and all(
                    getattr(getattr(p, "_kb_shadow", None), "_base", None) is buf for p in g):
                continue
            rows = sum(p.shape[0] for p in g)
            buf = torch.empty((rows, g[0].shape[1]), device=g[0].device, dtype=dtype)
            r = 0
            for p in g:
                p._kb_shadow = buf[r:r + p.shape[0]]  # type: ignore[attr-defined]
                p._kb_shadow_version = -1  # type: ignore[attr-defined]
                r += p.shape[0]
            self._fused[(gi, dtype)] = buf

    def fused(self, index: int, dtype: torch.dtype) -> torch.Tensor:
        """The stacked copy of fused group ``index`` (valid after ``get(dtype)``)."""

        return self._fused[(index, dtype)]

    def refresh(self) -> None:
        """Bring every 16-bit copy handed out so far up to date with its parameter."""

        for dtype in list(getattr(self, "_dtypes_seen", ())):
            self.get(dtype)

    def get(self, dtype: torch.dtype) -> Dict[int, torch.Tensor]:
        seen = self.__dict__.setdefault("_dtypes_seen", set())
        seen.add(dtype)
        if self.fused_groups:
            self._ensure_fused(dtype)
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


def accumulation_target(*params: torch.Tensor) -> Optional[torch.Tensor]:
    """The existing fp32 gradient buffer of ``params`` that a backward may add into directly, or None.

    Under gradient accumulation the second and later micro-steps would
    otherwise produce a fresh weight gradient that autograd then adds into
    ``.grad`` (one more read and write of every gradient). A backward may
    instead accumulate into ``.grad`` itself (a GEMM with the old gradient as
    its D operand) and return None for that weight, when nothing could
    observe the difference: gradients are not being recorded, every
    parameter already has a contiguous fp32 gradient of its own shape, no
    hook is registered on the parameters (a hook expects to see the
    accumulation), and -- for several parameters -- their gradients lie back
    to back in one buffer (the layout autograd keeps when it adopted the
    split views of one fused gradient on the first micro-step). Returns a
    [sum of rows, cols] view over those gradients.
    """

    if torch.is_grad_enabled() or not params:
        return None
    grads = []
    for p in params:
        g = p.grad
        if (g is None or g.dtype != torch.float32 or not g.is_contiguous() or g.shape != p.shape
                or p._backward_hooks or getattr(p, "_post_accumulate_grad_hooks", None)):
            return None
        grads.append(g)
    first = grads[0]
    cols = first.numel() // first.shape[0]
    rows = 0
    for g in grads:
        if (g.numel() // g.shape[0] != cols or g.untyped_storage().data_ptr() != first.untyped_storage().data_ptr()
                or g.data_ptr() != first.data_ptr() + rows * cols * 4):
            return None
        rows += g.shape[0]
    return first.as_strided((rows, cols), (cols, 1))
