"""GPT-2 decoder (124M "small" by default) on the native sm_100a kernels.

Parameter layout and names follow the usual GPT-2 module tree
(``transformer.wte/wpe/h.N.{ln_1,attn.c_attn,attn.c_proj,ln_2,mlp.c_fc,mlp.c_proj}/ln_f``,
``lm_head`` tied to ``wte``), with ``nn.Linear`` weights ``[out, in]``.

Execution under bf16/fp16 autocast on CUDA:

* one autograd node per transformer block (``_BlockFn``) whose forward and
  backward call the native kernels directly, so the residual stream stays
  fp32 (as autocast leaves it), bias + GELU and residual adds are fused into
  the GEMM epilogues, GELU's derivative is fused into the data-gradient GEMM of
  the MLP, and attention consumes the fused QKV output in place;
* the embedding is one gather kernel, and the final LayerNorm + tied LM head +
  cross-entropy are one node (``_HeadLossFn``) that never materialises fp32
  logits and overwrites the bf16 logits with their gradient in place.

Anywhere else (CPU, fp32) the same modules run the plain-PyTorch path, which
is also the numerical oracle of the tests.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import functional as kf
from ..utils.nn_utils import tag_param
from .common import LowPrecisionShadows, compute_dtype, to_lp


@dataclass
class GPT2Config:
    vocab_size: int = 50257
    block_size: int = 1024
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    layer_norm_eps: float = 1e-5
    init_std: float = 0.02


class CausalSelfAttention(nn.Module):
    def __init__(self, cfg: GPT2Config) -> None:
        super().__init__()
        self.n_head = cfg.n_head
        self.c_attn = nn.Linear(cfg.n_embd, 3 * cfg.n_embd)
        self.c_proj = nn.Linear(cfg.n_embd, cfg.n_embd)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, C = x.shape
        H = self.n_head
        q, k, v = self.c_attn(x).view(B, S, 3, H, C // H).unbind(2)
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        return self.c_proj(y.transpose(1, 2).reshape(B, S, C))


class MLP(nn.Module):
    def __init__(self, cfg: GPT2Config) -> None:
        super().__init__()
        self.c_fc = nn.Linear(cfg.n_embd, 4 * cfg.n_embd)
        self.c_proj = nn.Linear(4 * cfg.n_embd, cfg.n_embd)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.c_proj(F.gelu(self.c_fc(x), approximate="tanh"))


class Block(nn.Module):
    def __init__(self, cfg: GPT2Config) -> None:
        super().__init__()
        self.ln_1 = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_eps)
        self.attn = CausalSelfAttention(cfg)
        self.ln_2 = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_eps)
        self.mlp = MLP(cfg)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attn(self.ln_1(x))
        return x + self.mlp(self.ln_2(x))

    def matrices(self):
        return [self.attn.c_attn.weight, self.attn.c_proj.weight, self.mlp.c_fc.weight, self.mlp.c_proj.weight]


def _with_lp_copy(grad: torch.Tensor, lp: torch.Tensor) -> torch.Tensor:
    """Attach the low-precision copy of an fp32 residual-stream gradient.

    The LayerNorm backward kernel writes both copies in one pass; the next
    block's backward reuses the bf16 copy for its GEMMs instead of casting.
    """

    grad._kb_lp = lp  # type: ignore[attr-defined]
    return grad


def _lp_copy_of(grad: torch.Tensor, dtype: torch.dtype):
    lp = getattr(grad, "_kb_lp", None)
    if lp is None or lp.dtype != dtype or lp.numel() != grad.numel():
        return None
    return lp


class _BlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, ln1_w, ln1_b, attn_w, attn_b, proj_w, proj_b, ln2_w, ln2_b, fc_w, fc_b, fcp_w, fcp_b,
                lp, n_head, eps, causal=True):
        attn_w16, proj_w16, fc_w16, fcp_w16 = lp
        cdt = attn_w16.dtype
        B, S, C = x.shape
        M, H, D = B * S, n_head, C // n_head
        x2 = x.reshape(M, C)
        h1, m1, r1 = kf.norm_forward(x2, ln1_w, ln1_b, eps, rms=False, out_dtype=cdt)
        qkv = kf.gemm(h1, attn_w16, bias=attn_b)
        q5 = qkv.view(B, S, 3, H, D)
        a, lse = kf.flash_attention_forward(q5[:, :, 0], q5[:, :, 1], q5[:, :, 2], causal=causal)
        a2 = a.view(M, C)
        x_mid = kf.gemm(a2, proj_w16, bias=proj_b, d=x2, beta=1.0, out_dtype=torch.float32)
        h2, m2, r2 = kf.norm_forward(x_mid, ln2_w, ln2_b, eps, rms=False, out_dtype=cdt)
        pre = torch.empty((M, 4 * C), device=x.device, dtype=cdt)
        g = kf.gemm(h2, fc_w16, bias=fc_b, aux=pre, act=kf.ACT_GELU)
        out = kf.gemm(g, fcp_w16, bias=fcp_b, d=x_mid, beta=1.0, out_dtype=torch.float32)
        ctx.save_for_backward(x2, h1, m1, r1, qkv, a2, lse, x_mid, h2, m2, r2, pre, g, ln1_w, ln2_w,
                              attn_w16, proj_w16, fc_w16, fcp_w16)
        ctx.dims = (B, S, C, H, D)
        ctx.causal = causal
        return out.view(B, S, C)

    @staticmethod
    def backward(ctx, dout):
        (x2, h1, m1, r1, qkv, a2, lse, x_mid, h2, m2, r2, pre, g, ln1_w, ln2_w,
         attn_w16, proj_w16, fc_w16, fcp_w16) = ctx.saved_tensors
        B, S, C, H, D = ctx.dims
        M = B * S
        cdt = attn_w16.dtype
        dout2 = dout.reshape(M, C).float().contiguous()
        dy = _lp_copy_of(dout, cdt)
        dy = dy.reshape(M, C) if dy is not None else to_lp(dout2, cdt)
        # MLP
        dpre = kf.gemm(dy, fcp_w16, b_mn_major=True, d=pre, act=kf.ACT_GELU_BWD)
        d_fcp_w = kf.gemm(dy, g, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32)
        d_fcp_b = kf.bias_grad(dy)
        dh2 = kf.gemm(dpre, fc_w16, b_mn_major=True)
        d_fc_w = kf.gemm(dpre, h2, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32)
        d_fc_b = kf.bias_grad(dpre)
        dx_mid, d_ln2_w, d_ln2_b, dmid = kf.norm_backward(dh2, x_mid, ln2_w, m2, r2, rms=False, dres=dout2,
                                                          dx_dtype=torch.float32, want_lp=True)
        # attention output projection
        da = kf.gemm(dmid, proj_w16, b_mn_major=True)
        d_proj_w = kf.gemm(dmid, a2, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32)
        d_proj_b = kf.bias_grad(dmid)
        # attention
        q5 = qkv.view(B, S, 3, H, D)
        dqkv = torch.empty((B, S, 3, H, D), device=qkv.device, dtype=cdt)
        kf.flash_attention_backward(q5[:, :, 0], q5[:, :, 1], q5[:, :, 2], a2.view(B, S, H, D), da.view(B, S, H, D),
                                    lse, causal=ctx.causal, dq=dqkv[:, :, 0], dk=dqkv[:, :, 1], dv=dqkv[:, :, 2])
        dqkv2 = dqkv.view(M, 3 * C)
        dh1 = kf.gemm(dqkv2, attn_w16, b_mn_major=True)
        d_attn_w = kf.gemm(dqkv2, h1, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32)
        d_attn_b = kf.bias_grad(dqkv2)
        dx, d_ln1_w, d_ln1_b, dx_lp = kf.norm_backward(dh1, x2, ln1_w, m1, r1, rms=False, dres=dx_mid,
                                                       dx_dtype=torch.float32, want_lp=True)
        return (_with_lp_copy(dx.view(B, S, C), dx_lp), d_ln1_w, d_ln1_b, d_attn_w, d_attn_b, d_proj_w, d_proj_b, d_ln2_w, d_ln2_b,
                d_fc_w, d_fc_b, d_fcp_w, d_fcp_b, None, None, None, None)


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, wte, wpe):
        B, S = idx.shape
        out = kf.embedding_forward(idx, wte, wpe, S)
        ctx.save_for_backward(idx)
        ctx.meta = (wte.shape[0], wpe.shape[0], S)
        return out

    @staticmethod
    def backward(ctx, dout):
        (idx,) = ctx.saved_tensors
        V, P, S = ctx.meta
        dwte, dwpe = kf.embedding_backward(idx, dout.float().contiguous(), V, P, S)
        return None, dwte, dwpe


class _HeadLossFn(torch.autograd.Function):
    """Final LayerNorm + tied LM head + mean cross-entropy over non-ignored targets."""

    @staticmethod
    def forward(ctx, x, lnf_w, lnf_b, wte, wte16, targets, eps, ignore_index):
        B, S, C = x.shape
        M = B * S
        V = wte.shape[0]
        cdt = wte16.dtype
        x2 = x.reshape(M, C)
        h, m, r = kf.norm_forward(x2, lnf_w, lnf_b, eps, rms=False, out_dtype=cdt)
        vpad = (V + 63) // 64 * 64
        logits = torch.empty((M, vpad), device=x.device, dtype=cdt)
        kf.gemm(h, wte16, out=logits[:, :V])
        tgt = targets.reshape(-1)
        loss_rows, lse = kf.cross_entropy_forward(logits, tgt, V, ignore_index)
        n_valid = (tgt != ignore_index).sum().clamp_min(1).to(torch.float32)
        loss = loss_rows.sum() / n_valid
        ctx.save_for_backward(x2, h, m, r, logits, lse, tgt, n_valid, lnf_w, wte16)
        ctx.meta = (B, S, C, V, ignore_index)
        return loss

    @staticmethod
    def backward(ctx, dloss):
        x2, h, m, r, logits, lse, tgt, n_valid, lnf_w, wte16 = ctx.saved_tensors
        B, S, C, V, ignore_index = ctx.meta
        gscale = (dloss.float() / n_valid).reshape(1).contiguous()
        kf.cross_entropy_backward_(logits, tgt, lse, gscale, V, ignore_index)
        dlog = logits[:, :V]
        dh = kf.gemm(dlog, wte16, b_mn_major=True)
        dwte = kf.gemm(dlog, h, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32)
        dx, dlnf_w, dlnf_b, dx_lp = kf.norm_backward(dh, x2, lnf_w, m, r, rms=False, dx_dtype=torch.float32,
                                                     want_lp=True)
        return _with_lp_copy(dx.view(B, S, C), dx_lp), dlnf_w, dlnf_b, dwte, None, None, None, None


class GPT2(nn.Module):
    """GPT-2 language model. ``forward(idx, targets)`` returns the mean loss;
    ``forward(idx)`` returns logits (reference path only materialises them)."""

    def __init__(self, cfg: Optional[GPT2Config] = None, **overrides) -> None:
        super().__init__()
        cfg = cfg or GPT2Config()
        for k, v in overrides.items():
            setattr(cfg, k, v)
        self.config = cfg
        self.transformer = nn.ModuleDict(
            dict(
                wte=nn.Embedding(cfg.vocab_size, cfg.n_embd),
                wpe=nn.Embedding(cfg.block_size, cfg.n_embd),
                h=nn.ModuleList([Block(cfg) for _ in range(cfg.n_layer)]),
                ln_f=nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_eps),
            )
        )
        self.lm_head = nn.Linear(cfg.n_embd, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.transformer.wte.weight  # tied
        self._init_weights()
        # Muon takes the hidden matrices; embeddings, norms and biases use AdamW.
        for blk in self.transformer.h:
            for w in blk.matrices():
                tag_param(w, "wd")
        self._shadows = LowPrecisionShadows(
            [self.transformer.wte.weight] + [w for blk in self.transformer.h for w in blk.matrices()]
        )

    def _init_weights(self) -> None:
        std = self.config.init_std
        proj_std = std / math.sqrt(2 * self.config.n_layer)
        for name, mod in self.named_modules():
            if isinstance(mod, nn.Linear):
                nn.init.normal_(mod.weight, mean=0.0, std=proj_std if name.endswith("c_proj") else std)
                if mod.bias is not None:
                    nn.init.zeros_(mod.bias)
            elif isinstance(mod, nn.Embedding):
                nn.init.normal_(mod.weight, mean=0.0, std=std)

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None, ignore_index: int = -100):
        cdt = compute_dtype(idx.device)
        if cdt is None or targets is None:
            return self._forward_reference(idx, targets, ignore_index)
        tr = self.transformer
        eps = self.config.layer_norm_eps
        with torch.autocast("cuda", enabled=False):
            lp = self._shadows.get(cdt)
            x = _EmbeddingFn.apply(idx, tr.wte.weight, tr.wpe.weight)
            for blk in tr.h:
                w16 = tuple(lp[id(w)] for w in blk.matrices())
                x = _BlockFn.apply(
                    x, blk.ln_1.weight, blk.ln_1.bias, blk.attn.c_attn.weight, blk.attn.c_attn.bias,
                    blk.attn.c_proj.weight, blk.attn.c_proj.bias, blk.ln_2.weight, blk.ln_2.bias,
                    blk.mlp.c_fc.weight, blk.mlp.c_fc.bias, blk.mlp.c_proj.weight, blk.mlp.c_proj.bias,
                    w16, blk.attn.n_head, eps,
                )
            return _HeadLossFn.apply(x, tr.ln_f.weight, tr.ln_f.bias, tr.wte.weight, lp[id(tr.wte.weight)], targets,
                                     eps, ignore_index)

    def _forward_reference(self, idx, targets, ignore_index):
        B, S = idx.shape
        tr = self.transformer
        pos = torch.arange(S, device=idx.device)
        x = tr.wte(idx) + tr.wpe(pos)[None]
        for blk in tr.h:
            x = blk(x)
        x = tr.ln_f(x)
        logits = self.lm_head(x)
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1),
                               ignore_index=ignore_index)

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())
