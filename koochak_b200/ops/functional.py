"""Thin, shape-checked wrappers over the native kernels, with PyTorch references.

Every ``*_ref`` function is the plain-PyTorch definition of the same op in
fp32; tests compare the native kernels against them. The native wrappers
allocate their outputs (and scratch) from PyTorch's caching allocator so that
out-of-memory surfaces as ``torch.OutOfMemoryError``.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch
import torch.nn.functional as F

from ._ext import native

ACT_NONE, ACT_GELU, ACT_GELU_BWD = 0, 1, 2


# ----------------------------------------------------------------- GEMM


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a_mn_major: bool = False,
    b_mn_major: bool = False,
    out: Optional[torch.Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
    d: Optional[torch.Tensor] = None,
    alpha: float = 1.0,
    beta: float = 0.0,
    bias: Optional[torch.Tensor] = None,
    aux: Optional[torch.Tensor] = None,
    act: int = ACT_NONE,
    block_n: int = 0,
    symmetric: bool = False,
) -> torch.Tensor:
    """``out = epilogue(alpha * A @ B^T)`` on tcgen05 tensor cores.

    ``a`` is ``[.., M, K]`` (K-major) or, with ``a_mn_major``, ``[.., K, M]``.
    ``b`` is ``[.., N, K]`` or, with ``b_mn_major``, ``[.., K, N]``.
    Epilogue: ``+ bias[n]``; ``act=GELU`` stores the pre-activation to ``aux``
    and applies tanh-GELU; ``act=GELU_BWD`` multiplies by GELU'(d);
    otherwise ``+ beta * d``.

    ``symmetric=True`` declares the result symmetric (``X X^T``, or ``A A``
    plus ``beta * D`` with ``A`` and ``D`` symmetric; 16-bit output, no bias
    or activation): only the tiles on or above the diagonal are computed and
    the epilogue mirrors them, about half the work for large square outputs.
    Elements next to the diagonal may be written from both sides; both
    values are the same product up to rounding.
    """

    M = a.shape[-1] if a_mn_major else a.shape[-2]
    N = b.shape[-1] if b_mn_major else b.shape[-2]
    if out is None:
        shape = (*a.shape[:-2], M, N)
        out = torch.empty(shape, device=a.device, dtype=out_dtype or a.dtype)
    native().gemm(a, a_mn_major, b, b_mn_major, out, d, float(alpha), float(beta), bias, aux, int(act), int(block_n),
                  1 if symmetric else 0)
    return out


def gemm_ref(a, b, *, a_mn_major=False, b_mn_major=False, d=None, alpha=1.0, beta=0.0, bias=None, act=ACT_NONE):
    A = a.float().transpose(-1, -2) if a_mn_major else a.float()
    B = b.float().transpose(-1, -2) if b_mn_major else b.float()
    y = alpha * (A @ B.transpose(-1, -2))
    if bias is not None:
        y = y + bias.float()
    if act == ACT_GELU:
        return F.gelu(y, approximate="tanh"), y
    if act == ACT_GELU_BWD:
        h = d.float().detach().requires_grad_(True)
        with torch.enable_grad():
            g = torch.autograd.grad(F.gelu(h, approximate="tanh").sum(), h)[0]
        return y * g
    if d is not None and beta != 0.0:
        y = y + beta * d.float()
    return y


# ----------------------------------------------------------------- norms


def norm_forward(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], eps: float, *, rms: bool,
                 out_dtype: torch.dtype):
    rows = x.numel() // x.shape[-1]
    y = torch.empty(x.shape, device=x.device, dtype=out_dtype)
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    mean = None if rms else torch.empty(rows, device=x.device, dtype=torch.float32)
    native().norm_forward(x, weight, bias, y, mean, rstd, float(eps), bool(rms))
    return y, mean, rstd


def norm_backward(dy, x, weight, mean, rstd, *, rms: bool, dres: Optional[torch.Tensor] = None,
                  dx_dtype: Optional[torch.dtype] = None, need_bias_grad: bool = True, want_lp: bool = False):
    """Returns (dx, dweight, dbias[, dx in dy's dtype when ``want_lp``])."""

    C = x.shape[-1]
    rows = x.numel() // C
    dx = torch.empty(x.shape, device=x.device, dtype=dx_dtype or (dres.dtype if dres is not None else x.dtype))
    dw = torch.empty(C, device=x.device, dtype=torch.float32)
    db = None if (rms or not need_bias_grad) else torch.empty(C, device=x.device, dtype=torch.float32)
    ws = torch.empty(native().norm_backward_workspace_elems(rows, C, x.device.index or 0), device=x.device,
                     dtype=torch.float32)
    lp = torch.empty(x.shape, device=x.device, dtype=dy.dtype) if want_lp else None
    native().norm_backward(dy, x, weight, mean, rstd, dres, dx, dw, db, ws, bool(rms), False, lp)
    if want_lp:
        return dx, dw, db, lp
    return dx, dw, db


def layer_norm_ref(x, w, b, eps):
    return F.layer_norm(x.float(), (x.shape[-1],), w.float(), None if b is None else b.float(), eps)


def rms_norm_ref(x, w, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


# ----------------------------------------------------------------- attention


def flash_attention_forward(q, k, v, *, causal: bool, scale: Optional[float] = None, out=None):
    """q, k, v: [B, S, H, D] views (token stride free). Returns (o, lse[B, H, S])."""

    B, S, H, D = q.shape
    scale = (1.0 / math.sqrt(D)) if scale is None else scale
    if out is None:
        out = torch.empty((B, S, H, D), device=q.device, dtype=q.dtype)
    lse = torch.empty((B, H, S), device=q.device, dtype=torch.float32)
    native().flash_attention_forward(q, k, v, out, lse, float(scale), bool(causal))
    return out, lse


def flash_attention_backward(q, k, v, o, do, lse, *, causal: bool, scale: Optional[float] = None, dq=None, dk=None,
                             dv=None):
    B, S, H, D = q.shape
    scale = (1.0 / math.sqrt(D)) if scale is None else scale
    dq = torch.empty_like(q, memory_format=torch.contiguous_format) if dq is None else dq
    dk = torch.empty_like(k, memory_format=torch.contiguous_format) if dk is None else dk
    dv = torch.empty_like(v, memory_format=torch.contiguous_format) if dv is None else dv
    ws = torch.empty(B * S * H * D + B * H * S, device=q.device, dtype=torch.float32)
    native().flash_attention_backward(q, k, v, o, do, lse, dq, dk, dv, ws, float(scale), bool(causal))
    return dq, dk, dv


def attention_ref(q, k, v, *, causal: bool, scale: Optional[float] = None):
    """[B, S, H, D] inputs, fp32 math."""

    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    o = F.scaled_dot_product_attention(qf, kf, vf, is_causal=causal, scale=scale)
    return o.transpose(1, 2)


# ----------------------------------------------------------------- misc


def embedding_forward(idx, wte, wpe, seq_len):
    out = torch.empty((*idx.shape, wte.shape[1]), device=idx.device, dtype=torch.float32)
    native().embedding_forward(idx.contiguous(), wte, wpe, out, int(seq_len))
    return out


def embedding_backward(idx, dout, vocab, wpe_rows, seq_len, want_wpe=True):
    C = dout.shape[-1]
    dwte = torch.zeros((vocab, C), device=dout.device, dtype=torch.float32)
    dwpe = torch.zeros((wpe_rows, C), device=dout.device, dtype=torch.float32) if want_wpe else None
    native().embedding_backward(idx.contiguous(), dout.contiguous(), dwte, dwpe, int(seq_len))
    return dwte, dwpe


def cross_entropy_forward(logits, target, vocab, ignore_index=-100):
    rows = target.numel()
    loss = torch.empty(rows, device=logits.device, dtype=torch.float32)
    lse = torch.empty(rows, device=logits.device, dtype=torch.float32)
    native().cross_entropy_forward(logits, target.reshape(-1).contiguous(), loss, lse, int(vocab), int(ignore_index))
    return loss, lse


def cross_entropy_backward_(logits, target, lse, gscale, vocab, ignore_index=-100):
    native().cross_entropy_backward(logits, target.reshape(-1).contiguous(), lse, gscale, int(vocab), int(ignore_index))
    return logits


def bias_grad(g: torch.Tensor) -> torch.Tensor:
    """Column sums of ``g`` in fp32 (the bias gradient), deterministic (two passes, no atomics)."""

    out = torch.empty(g.shape[-1], device=g.device, dtype=torch.float32)
    native().bias_grad(g, out, False)
    return out


def cast_multi(src: Sequence[torch.Tensor], dst: Sequence[torch.Tensor]) -> None:
    native().cast_multi(list(src), list(dst))


def swiglu_forward(gu):
    F_ = gu.shape[-1] // 2
    h = torch.empty((*gu.shape[:-1], F_), device=gu.device, dtype=gu.dtype)
    native().swiglu_forward(gu, h)
    return h


def swiglu_backward(gu, dh):
    dgu = torch.empty_like(gu)
    native().swiglu_backward(gu, dh, dgu)
    return dgu


def swiglu_ref(gu):
    g, u = gu.float().chunk(2, dim=-1)
    return F.silu(g) * u


def patchify(images, patch: int, dtype: torch.dtype):
    """fp32 NCHW images -> [B * patches, C * patch * patch] rows in ``dtype`` (Conv2d weight column order)."""

    B, C, H, W = images.shape
    out = torch.empty((B * (H // patch) * (W // patch), C * patch * patch), device=images.device, dtype=dtype)
    native().patchify(images.contiguous(), out, int(patch))
    return out


def patchify_ref(images, patch: int):
    B, C, H, W = images.shape
    x = images.reshape(B, C, H // patch, patch, W // patch, patch)
    return x.permute(0, 2, 4, 1, 3, 5).reshape(B * (H // patch) * (W // patch), C * patch * patch)


def rope_apply_(x, cos, sin, inverse=False):
    B, S, H, D = x.shape
    native().rope_apply(x, cos, sin, S, H, D, bool(inverse))
    return x


def rope_ref(x, cos, sin):
    """x: [B, S, H, D]; cos/sin: [S, D/2]. Rotate-half convention."""

    xf = x.float()
    half = xf.shape[-1] // 2
    x1, x2 = xf[..., :half], xf[..., half:]
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
