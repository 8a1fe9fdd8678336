"""ViT-B/16 image classifier on the native sm_100a kernels.

Shape of the default config: 224 x 224 x 3 inputs, 16 x 16 patches (196
tokens + a class token), 12 pre-LayerNorm blocks of width 768 with 12 heads,
MLP 3072 (GELU), 1000 classes. Parameter names follow the common ViT layout
(``patch_embed.proj``, ``cls_token``, ``pos_embed``, ``blocks.N``, ``norm``,
``head``). The blocks reuse the GPT-2 block node with non-causal attention,
so bias + GELU and residual adds are fused into GEMM epilogues and attention
runs on the flash kernel (S = 197).

Under fp16 (or bf16) autocast on CUDA: the patch extraction is one kernel
writing 16-bit rows in the Conv2d weight's column order, the patch embedding
one GEMM with the bias fused; class token and position embedding are added
in fp32. With fp16 the GradScaler path (unscale, finite check, skip step) is
exercised. Elsewhere the plain-PyTorch path runs (the numerical oracle).
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
from .common import LowPrecisionShadows, compute_dtype
from .gpt2 import Block, GPT2Config, _BlockFn

__all__ = ["ViTConfig", "ViT"]


@dataclass
class ViTConfig:
    image_size: int = 224
    patch_size: int = 16
    in_chans: int = 3
    num_classes: int = 1000
    dim: int = 768
    depth: int = 12
    n_head: int = 12
    mlp_ratio: int = 4
    norm_eps: float = 1e-6
    init_std: float = 0.02


class PatchEmbed(nn.Module):
    def __init__(self, cfg: ViTConfig) -> None:
        super().__init__()
        self.patch = cfg.patch_size
        self.proj = nn.Conv2d(cfg.in_chans, cfg.dim, cfg.patch_size, stride=cfg.patch_size)

    def forward(self, x):
        return self.proj(x).flatten(2).transpose(1, 2)


class _PatchEmbedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, images, weight, bias, w16, patch):
        rows = kf.patchify(images, patch, w16.dtype)
        out = kf.gemm(rows, w16, bias=bias, out_dtype=torch.float32)
        ctx.save_for_backward(rows)
        return out

    @staticmethod
    def backward(ctx, dout):
        (rows,) = ctx.saved_tensors
        d16 = dout.to(rows.dtype).contiguous()
        dW = kf.gemm(d16, rows, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32)
        db = kf.bias_grad(d16)
        return None, dW, db, None, None


class ViT(nn.Module):
    """``forward(images, labels)`` returns the mean loss; ``forward(images)`` returns logits."""

    def __init__(self, cfg: Optional[ViTConfig] = None, **overrides) -> None:
        super().__init__()
        cfg = cfg or ViTConfig()
        for k, v in overrides.items():
            setattr(cfg, k, v)
        self.config = cfg
        n_tok = (cfg.image_size // cfg.patch_size) ** 2 + 1
        self.patch_embed = PatchEmbed(cfg)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, cfg.dim))
        self.pos_embed = nn.Parameter(torch.zeros(1, n_tok, cfg.dim))
        bcfg = GPT2Config(n_embd=cfg.dim, n_head=cfg.n_head, layer_norm_eps=cfg.norm_eps)
        self.blocks = nn.ModuleList([Block(bcfg) for _ in range(cfg.depth)])
        self.norm = nn.LayerNorm(cfg.dim, eps=cfg.norm_eps)
        self.head = nn.Linear(cfg.dim, cfg.num_classes)
        self._init_weights()
        for blk in self.blocks:
            for w in blk.matrices():
                tag_param(w, "wd")
        self._shadows = LowPrecisionShadows([self.patch_embed.proj.weight] +
                                            [w for blk in self.blocks for w in blk.matrices()])

    def _init_weights(self) -> None:
        std = self.config.init_std
        nn.init.normal_(self.pos_embed, std=std)
        nn.init.normal_(self.cls_token, std=1e-6)
        for mod in self.modules():
            if isinstance(mod, nn.Linear):
                nn.init.trunc_normal_(mod.weight, std=std)
                if mod.bias is not None:
                    nn.init.zeros_(mod.bias)
        w = self.patch_embed.proj.weight
        nn.init.trunc_normal_(w, std=math.sqrt(1.0 / w[0].numel()))
        nn.init.zeros_(self.patch_embed.proj.bias)

    def _tokens_native(self, images, lp):
        B = images.shape[0]
        cfg = self.config
        w = self.patch_embed.proj.weight
        w2 = w.view(w.shape[0], -1)
        w16 = lp[id(w)].view(w.shape[0], -1)
        pe = _PatchEmbedFn.apply(images, w2, self.patch_embed.proj.bias, w16, cfg.patch_size)
        pe = pe.view(B, -1, cfg.dim)
        return torch.cat([self.cls_token.expand(B, -1, -1), pe], dim=1) + self.pos_embed

    def forward(self, images: torch.Tensor, labels: Optional[torch.Tensor] = None):
        cdt = compute_dtype(images.device)
        if cdt is None:
            return self._forward_reference(images, labels)
        eps = self.config.norm_eps
        with torch.autocast("cuda", enabled=False):
            lp = self._shadows.get(cdt)
            x = self._tokens_native(images.float(), lp)
            for blk in self.blocks:
                w16 = tuple(lp[id(w)] for w in blk.matrices())
                x = _BlockFn.apply(
                    x, blk.ln_1.weight, blk.ln_1.bias, blk.attn.c_attn.weight, blk.attn.c_attn.bias,
                    blk.attn.c_proj.weight, blk.attn.c_proj.bias, blk.ln_2.weight, blk.ln_2.bias,
                    blk.mlp.c_fc.weight, blk.mlp.c_fc.bias, blk.mlp.c_proj.weight, blk.mlp.c_proj.bias,
                    w16, blk.attn.n_head, eps, False,
                )
            cls = F.layer_norm(x[:, 0], (self.config.dim,), self.norm.weight, self.norm.bias, eps)
            logits = F.linear(cls, self.head.weight, self.head.bias)
            if labels is None:
                return logits
            return F.cross_entropy(logits, labels)

    def _forward_reference(self, images, labels):
        B = images.shape[0]
        x = self.patch_embed(images)
        x = torch.cat([self.cls_token.expand(B, -1, -1), x], dim=1) + self.pos_embed
        for blk in self.blocks:
            x = self._block_ref(blk, x)
        logits = self.head(self.norm(x)[:, 0])
        if labels is None:
            return logits
        return F.cross_entropy(logits.float(), labels)

    @staticmethod
    def _block_ref(blk, x):
        B, S, C = x.shape
        H = blk.attn.n_head
        q, k, v = blk.attn.c_attn(blk.ln_1(x)).view(B, S, 3, H, C // H).unbind(2)
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=False)
        x = x + blk.attn.c_proj(y.transpose(1, 2).reshape(B, S, C))
        return x + blk.mlp(blk.ln_2(x))

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())
