"""Llama-style decoder (1.3B by default) on the native sm_100a kernels.

Shape of the default config: 24 layers, d=2048, 16 heads of 128, RMSNorm,
rotary position embeddings (rotate-half convention, theta 10000), SwiGLU MLP
with FFN 5504, vocab 32000, untied embedding and LM head, no biases.
Parameter names follow the common Llama module tree
(``model.embed_tokens``, ``model.layers.N.{input_layernorm,
self_attn.{q,k,v,o}_proj, post_attention_layernorm, mlp.{gate,up,down}_proj}``,
``model.norm``, ``lm_head``).

Under bf16/fp16 autocast on CUDA each layer is one autograd node
(``_LayerFn``):

* RMSNorm forward/backward kernels (the backward also writes the bf16 copy of
  the residual gradient the next layer's GEMMs consume);
* q, k and v stay separate parameters (Muon orthogonalises each) but their
  bf16 copies are row blocks of one buffer, so the projection is one GEMM;
  RoPE rotates q and k in place inside that output and attention reads it
  without a copy; the backward applies the inverse rotation to dq and dk;
* gate and up projections write the two halves of one [M, 2F] buffer, SwiGLU
  reads it; the residual adds are fused into the o_proj / down_proj GEMM
  epilogues (fp32 residual stream).

Elsewhere the same modules run plain PyTorch, the oracle of the tests.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import functional as kf
from ..ops._ext import native
from ..utils.nn_utils import tag_param
from .common import LowPrecisionShadows, accumulation_target, compute_dtype, to_lp
from .gpt2 import _lp_copy_of, _with_lp_copy

__all__ = ["LlamaConfig", "Llama", "rope_tables"]


@dataclass
class LlamaConfig:
    vocab_size: int = 32000
    max_seq_len: int = 2048
    n_layer: int = 24
    n_head: int = 16
    dim: int = 2048
    ffn_dim: int = 5504
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    init_std: float = 0.02


def rope_tables(seq_len: int, head_dim: int, theta: float, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos, sin of shape [seq_len, head_dim / 2] (fp32)."""

    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = torch.arange(seq_len, dtype=torch.float64)[:, None] * inv[None, :]
    return ang.cos().float().to(device), ang.sin().float().to(device)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight).to(x.dtype)


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        self.n_head = cfg.n_head
        self.q_proj = nn.Linear(cfg.dim, cfg.dim, bias=False)
        self.k_proj = nn.Linear(cfg.dim, cfg.dim, bias=False)
        self.v_proj = nn.Linear(cfg.dim, cfg.dim, bias=False)
        self.o_proj = nn.Linear(cfg.dim, cfg.dim, bias=False)

    def forward(self, x, cos, sin):
        B, S, C = x.shape
        H = self.n_head
        D = C // H
        q = kf.rope_ref(self.q_proj(x).view(B, S, H, D), cos, sin).to(x.dtype)
        k = kf.rope_ref(self.k_proj(x).view(B, S, H, D), cos, sin).to(x.dtype)
        v = self.v_proj(x).view(B, S, H, D)
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        return self.o_proj(y.transpose(1, 2).reshape(B, S, C))


class FeedForward(nn.Module):
    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(cfg.dim, cfg.ffn_dim, bias=False)
        self.up_proj = nn.Linear(cfg.dim, cfg.ffn_dim, bias=False)
        self.down_proj = nn.Linear(cfg.ffn_dim, cfg.dim, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.self_attn = Attention(cfg)
        self.post_attention_layernorm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.mlp = FeedForward(cfg)

    def forward(self, x, cos, sin):
        x = x + self.self_attn(self.input_layernorm(x), cos, sin)
        return x + self.mlp(self.post_attention_layernorm(x))

    def matrices(self):
        a, m = self.self_attn, self.mlp
        return [a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, a.o_proj.weight, m.gate_proj.weight,
                m.up_proj.weight, m.down_proj.weight]


def _wgrad(a: torch.Tensor, b: torch.Tensor, *weights: torch.Tensor) -> Optional[torch.Tensor]:
    """fp32 weight gradient a^T b (both operands token-major) of ``weights`` (stacked by rows).

    Added straight into the weights' ``.grad`` when ``accumulation_target``
    allows it (later micro-steps of gradient accumulation; None is then
    returned, so autograd adds nothing), else returned for autograd.
    """

    tgt = accumulation_target(*weights)
    if tgt is not None:
        kf.gemm(a, b, a_mn_major=True, b_mn_major=True, out=tgt, d=tgt, beta=1.0)
        return None
    return kf.gemm(a, b, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32)


class _LayerFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_in, w_post, wq, wk, wv, wo, wg, wu, wd, lp, cos, sin, n_head, eps):
        qkv_w16, o_w16, gu_w16, down_w16 = lp
        cdt = o_w16.dtype
        B, S, C = x.shape
        M, H, D = B * S, n_head, C // n_head
        Fd = gu_w16.shape[0] // 2
        x2 = x.reshape(M, C)
        h1, _, r1 = kf.norm_forward(x2, w_in, None, eps, rms=True, out_dtype=cdt)
        qkv = kf.gemm(h1, qkv_w16)
        q5 = qkv.view(B, S, 3, H, D)
        kf.rope_apply_(q5[:, :, :2].view(B, S, 2 * H, D), cos, sin)  # q and k heads: one launch
        a, lse = kf.flash_attention_forward(q5[:, :, 0], q5[:, :, 1], q5[:, :, 2], causal=True)
        a2 = a.view(M, C)
        x_mid = kf.gemm(a2, o_w16, d=x2, beta=1.0, out_dtype=torch.float32)
        h2, _, r2 = kf.norm_forward(x_mid, w_post, None, eps, rms=True, out_dtype=cdt)
        gu = kf.gemm(h2, gu_w16)                      # [M, 2F]: gate | up
        hs = kf.swiglu_forward(gu)                     # [M, F]
        out = kf.gemm(hs, down_w16, d=x_mid, beta=1.0, out_dtype=torch.float32)
        ctx.save_for_backward(x2, h1, r1, qkv, a2, lse, x_mid, h2, r2, gu, hs, w_in, w_post, qkv_w16, o_w16, gu_w16,
                              down_w16, cos, sin)
        ctx.dims = (B, S, C, H, D, Fd)
        ctx.weights = (wq, wk, wv, wo, wg, wu, wd)
        return out.view(B, S, C)

    @staticmethod
    def backward(ctx, dout):
        (x2, h1, r1, qkv, a2, lse, x_mid, h2, r2, gu, hs, w_in, w_post, qkv_w16, o_w16, gu_w16, down_w16, cos,
         sin) = ctx.saved_tensors
        B, S, C, H, D, Fd = ctx.dims
        M = B * S
        cdt = o_w16.dtype
        dout2 = dout.reshape(M, C).float().contiguous()
        dy = _lp_copy_of(dout, cdt)
        dy = dy.reshape(M, C) if dy is not None else to_lp(dout2, cdt)
        # MLP
        wq, wk, wv, wo, wg, wu, wd = ctx.weights
        dhs = kf.gemm(dy, down_w16, b_mn_major=True)
        d_down = _wgrad(dy, hs, wd)
        dgu = kf.swiglu_backward(gu, dhs)
        dh2 = kf.gemm(dgu, gu_w16, b_mn_major=True)
        d_gu = _wgrad(dgu, h2, wg, wu)
        dx_mid, d_post, _, dmid = kf.norm_backward(dh2, x_mid, w_post, None, r2, rms=True, dres=dout2,
                                                   dx_dtype=torch.float32, want_lp=True)
        # attention
        da = kf.gemm(dmid, o_w16, b_mn_major=True)
        d_o = _wgrad(dmid, a2, wo)
        q5 = qkv.view(B, S, 3, H, D)
        dqkv = torch.empty((B, S, 3, H, D), device=qkv.device, dtype=cdt)
        kf.flash_attention_backward(q5[:, :, 0], q5[:, :, 1], q5[:, :, 2], a2.view(B, S, H, D), da.view(B, S, H, D),
                                    lse, causal=True, dq=dqkv[:, :, 0], dk=dqkv[:, :, 1], dv=dqkv[:, :, 2])
        kf.rope_apply_(dqkv[:, :, :2].view(B, S, 2 * H, D), cos, sin, inverse=True)
        dqkv2 = dqkv.view(M, 3 * C)
        dh1 = kf.gemm(dqkv2, qkv_w16, b_mn_major=True)
        d_qkv = _wgrad(dqkv2, h1, wq, wk, wv)
        dx, d_in, _, dx_lp = kf.norm_backward(dh1, x2, w_in, None, r1, rms=True, dres=dx_mid,
                                              dx_dtype=torch.float32, want_lp=True)
        dq, dk, dv = d_qkv.split(C, dim=0) if d_qkv is not None else (None, None, None)
        dg, du = d_gu.split(Fd, dim=0) if d_gu is not None else (None, None)
        return (_with_lp_copy(dx.view(B, S, C), dx_lp), d_in, d_post, dq, dk, dv, d_o, dg, du, d_down,
                None, None, None, None, None)


class _EmbedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, w):
        ctx.save_for_backward(idx)
        ctx.rows = w.shape[0]
        ctx.weight = w
        return kf.embedding_forward(idx, w, None, idx.shape[1])

    @staticmethod
    def backward(ctx, dout):
        (idx,) = ctx.saved_tensors
        tgt = accumulation_target(ctx.weight)
        if tgt is not None:  # scatter-add straight into the existing gradient
            native().embedding_backward(idx.contiguous(), dout.float().contiguous(), tgt, None, int(idx.shape[1]))
            return None, None
        dw, _ = kf.embedding_backward(idx, dout.float().contiguous(), ctx.rows, 0, idx.shape[1], want_wpe=False)
        return None, dw


class _HeadFn(torch.autograd.Function):
    """Final RMSNorm + LM head + mean cross-entropy (bf16 logits, gradient written in place)."""

    @staticmethod
    def forward(ctx, x, norm_w, head_w, head_w16, targets, eps, ignore_index):
        B, S, C = x.shape
        M, V = B * S, head_w.shape[0]
        cdt = head_w16.dtype
        x2 = x.reshape(M, C)
        h, _, r = kf.norm_forward(x2, norm_w, None, eps, rms=True, out_dtype=cdt)
        vpad = (V + 63) // 64 * 64
        logits = torch.empty((M, vpad), device=x.device, dtype=cdt)
        kf.gemm(h, head_w16, out=logits[:, :V])
        tgt = targets.reshape(-1)
        loss_rows, lse = kf.cross_entropy_forward(logits, tgt, V, ignore_index)
        n_valid = (tgt != ignore_index).sum().clamp_min(1).to(torch.float32)
        ctx.save_for_backward(x2, h, r, logits, lse, tgt, n_valid, norm_w, head_w16)
        ctx.meta = (B, S, C, V, ignore_index, eps)
        ctx.head_weight = head_w
        return loss_rows.sum() / n_valid

    @staticmethod
    def backward(ctx, dloss):
        x2, h, r, logits, lse, tgt, n_valid, norm_w, head_w16 = ctx.saved_tensors
        B, S, C, V, ignore_index, eps = ctx.meta
        kf.cross_entropy_backward_(logits, tgt, lse, (dloss.float() / n_valid).reshape(1).contiguous(), V,
                                   ignore_index)
        dlog = logits[:, :V]
        dh = kf.gemm(dlog, head_w16, b_mn_major=True)
        dW = _wgrad(dlog, h, ctx.head_weight)
        dx, dnorm, _, dx_lp = kf.norm_backward(dh, x2, norm_w, None, r, rms=True, dx_dtype=torch.float32,
                                               want_lp=True)
        return _with_lp_copy(dx.view(B, S, C), dx_lp), dnorm, dW, None, None, None, None


class _Model(nn.Module):
    def __init__(self, cfg: LlamaConfig) -> None:
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.dim)
        self.layers = nn.ModuleList([DecoderLayer(cfg) for _ in range(cfg.n_layer)])
        self.norm = RMSNorm(cfg.dim, cfg.norm_eps)


class Llama(nn.Module):
    """``forward(idx, targets)`` returns the mean loss; ``forward(idx)`` returns logits (reference path)."""

    def __init__(self, cfg: Optional[LlamaConfig] = None, **overrides) -> None:
        super().__init__()
        cfg = cfg or LlamaConfig()
        for k, v in overrides.items():
            setattr(cfg, k, v)
        if cfg.dim % cfg.n_head or (cfg.dim // cfg.n_head) not in (64, 128):
            raise ValueError("head dimension must be 64 or 128")
        self.config = cfg
        self.model = _Model(cfg)
        self.lm_head = nn.Linear(cfg.dim, cfg.vocab_size, bias=False)
        self._init_weights()
        for layer in self.model.layers:
            for w in layer.matrices():
                tag_param(w, "wd")
        mats = [w for layer in self.model.layers for w in layer.matrices()]
        groups = []
        for layer in self.model.layers:
            a, m = layer.self_attn, layer.mlp
            groups += [[a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], [m.gate_proj.weight, m.up_proj.weight]]
        self._shadows = LowPrecisionShadows([self.lm_head.weight] + mats, fused_groups=groups)
        self._rope: Dict[tuple, Tuple[torch.Tensor, torch.Tensor]] = {}

    def _init_weights(self) -> None:
        std = self.config.init_std
        out_std = std / math.sqrt(2 * self.config.n_layer)
        for name, mod in self.named_modules():
            if isinstance(mod, nn.Linear):
                nn.init.normal_(mod.weight, 0.0, out_std if name.endswith(("o_proj", "down_proj")) else std)
            elif isinstance(mod, nn.Embedding):
                nn.init.normal_(mod.weight, 0.0, std)

    def rope(self, S: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        key = (S, str(device))
        if key not in self._rope:
            D = self.config.dim // self.config.n_head
            self._rope[key] = rope_tables(S, D, self.config.rope_theta, device)
        return self._rope[key]

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None, ignore_index: int = -100):
        cdt = compute_dtype(idx.device)
        B, S = idx.shape
        cos, sin = self.rope(S, idx.device)
        if cdt is None or targets is None:
            return self._forward_reference(idx, targets, ignore_index, cos, sin)
        cfg = self.config
        with torch.autocast("cuda", enabled=False):
            lp = self._shadows.get(cdt)
            x = _EmbedFn.apply(idx, self.model.embed_tokens.weight)
            gi = 0
            for layer in self.model.layers:
                a, m = layer.self_attn, layer.mlp
                w16 = (self._shadows.fused(gi, cdt), lp[id(a.o_proj.weight)], self._shadows.fused(gi + 1, cdt),
                       lp[id(m.down_proj.weight)])
                gi += 2
                x = _LayerFn.apply(x, layer.input_layernorm.weight, layer.post_attention_layernorm.weight,
                                   a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, a.o_proj.weight,
                                   m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight, w16, cos, sin,
                                   cfg.n_head, cfg.norm_eps)
            return _HeadFn.apply(x, self.model.norm.weight, self.lm_head.weight, lp[id(self.lm_head.weight)],
                                 targets, cfg.norm_eps, ignore_index)

    def _forward_reference(self, idx, targets, ignore_index, cos, sin):
        x = self.model.embed_tokens(idx)
        for layer in self.model.layers:
            x = layer(x, cos, sin)
        logits = self.lm_head(self.model.norm(x))
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1),
                               ignore_index=ignore_index)

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())
