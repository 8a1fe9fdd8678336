"""Plain-PyTorch benchmark models for the reference arm of bench.py.

These are the "user workloads" the reference framework is driven with: stock
``nn.Linear`` (cuBLAS), ``F.scaled_dot_product_attention`` and
``nn.LayerNorm`` modules, with no code from koochak_b200. Shapes match the
koochak_b200 models so both arms train the same architecture.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class _Attn(nn.Module):
    def __init__(self, d: int, h: int, causal: bool = True) -> None:
        super().__init__()
        self.h = h
        self.causal = causal
        self.c_attn = nn.Linear(d, 3 * d)
        self.c_proj = nn.Linear(d, d)

    def forward(self, x):
        B, S, C = x.shape
        q, k, v = self.c_attn(x).view(B, S, 3, self.h, C // self.h).unbind(2)
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=self.causal)
        return self.c_proj(y.transpose(1, 2).reshape(B, S, C))


class _Block(nn.Module):
    def __init__(self, d: int, h: int, causal: bool = True, eps: float = 1e-5) -> None:
        super().__init__()
        self.ln_1 = nn.LayerNorm(d, eps=eps)
        self.attn = _Attn(d, h, causal)
        self.ln_2 = nn.LayerNorm(d, eps=eps)
        self.c_fc = nn.Linear(d, 4 * d)
        self.c_proj = nn.Linear(4 * d, d)

    def forward(self, x):
        x = x + self.attn(self.ln_1(x))
        return x + self.c_proj(F.gelu(self.c_fc(self.ln_2(x)), approximate="tanh"))

    def matrices(self):
        return [self.attn.c_attn.weight, self.attn.c_proj.weight, self.c_fc.weight, self.c_proj.weight]


class PlainGPT2(nn.Module):
    """GPT-2 small by default: 12 layers, d=768, 12 heads, vocab 50257, block 1024, tied head."""

    def __init__(self, n_layer: int = 12, n_head: int = 12, n_embd: int = 768, vocab_size: int = 50257,
                 block_size: int = 1024) -> None:
        super().__init__()
        self.wte = nn.Embedding(vocab_size, n_embd)
        self.wpe = nn.Embedding(block_size, n_embd)
        self.blocks = nn.ModuleList([_Block(n_embd, n_head) for _ in range(n_layer)])
        self.ln_f = nn.LayerNorm(n_embd)
        self.lm_head = nn.Linear(n_embd, vocab_size, bias=False)
        self.lm_head.weight = self.wte.weight
        for name, m in self.named_modules():
            if isinstance(m, nn.Linear):
                std = 0.02 / math.sqrt(2 * n_layer) if name.endswith("c_proj") else 0.02
                nn.init.normal_(m.weight, std=std)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, std=0.02)

    def forward(self, idx, targets=None):
        B, S = idx.shape
        x = self.wte(idx) + self.wpe(torch.arange(S, device=idx.device))[None]
        for blk in self.blocks:
            x = blk(x)
        logits = self.lm_head(self.ln_f(x))
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().view(-1, logits.size(-1)), targets.reshape(-1))


class _LlamaLayer(nn.Module):
    def __init__(self, d: int, h: int, ffn: int, eps: float) -> None:
        super().__init__()
        self.h = h
        self.input_layernorm = nn.RMSNorm(d, eps=eps)
        self.q_proj = nn.Linear(d, d, bias=False)
        self.k_proj = nn.Linear(d, d, bias=False)
        self.v_proj = nn.Linear(d, d, bias=False)
        self.o_proj = nn.Linear(d, d, bias=False)
        self.post_attention_layernorm = nn.RMSNorm(d, eps=eps)
        self.gate_proj = nn.Linear(d, ffn, bias=False)
        self.up_proj = nn.Linear(d, ffn, bias=False)
        self.down_proj = nn.Linear(ffn, d, bias=False)

    @staticmethod
    def _rope(x, cos, sin):
        half = x.shape[-1] // 2
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)

    def forward(self, x, cos, sin):
        B, S, C = x.shape
        D = C // self.h
        h = self.input_layernorm(x)
        q = self._rope(self.q_proj(h).view(B, S, self.h, D).transpose(1, 2), cos, sin)
        k = self._rope(self.k_proj(h).view(B, S, self.h, D).transpose(1, 2), cos, sin)
        v = self.v_proj(h).view(B, S, self.h, D).transpose(1, 2)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.o_proj(y.transpose(1, 2).reshape(B, S, C))
        h = self.post_attention_layernorm(x)
        return x + self.down_proj(F.silu(self.gate_proj(h)) * self.up_proj(h))

    def matrices(self):
        return [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.o_proj.weight,
                self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight]


class PlainLlama(nn.Module):
    """Llama-style 1.3B by default: 24 layers, d=2048, 16 heads, RMSNorm, RoPE, SwiGLU 5504, vocab 32000."""

    def __init__(self, n_layer: int = 24, n_head: int = 16, dim: int = 2048, ffn: int = 5504, vocab_size: int = 32000,
                 eps: float = 1e-5, theta: float = 10000.0) -> None:
        super().__init__()
        self.n_head, self.dim, self.theta = n_head, dim, theta
        self.embed_tokens = nn.Embedding(vocab_size, dim)
        self.layers = nn.ModuleList([_LlamaLayer(dim, n_head, ffn, eps) for _ in range(n_layer)])
        self.norm = nn.RMSNorm(dim, eps=eps)
        self.lm_head = nn.Linear(dim, vocab_size, bias=False)
        for name, m in self.named_modules():
            if isinstance(m, nn.Linear):
                std = 0.02 / math.sqrt(2 * n_layer) if name.endswith(("o_proj", "down_proj")) else 0.02
                nn.init.normal_(m.weight, std=std)
            elif isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, std=0.02)

    def blocks_matrices(self):
        return [w for layer in self.layers for w in layer.matrices()]

    def forward(self, idx, targets=None):
        B, S = idx.shape
        D = self.dim // self.n_head
        inv = 1.0 / (self.theta ** (torch.arange(0, D, 2, device=idx.device, dtype=torch.float32) / D))
        ang = torch.arange(S, device=idx.device, dtype=torch.float32)[:, None] * inv[None]
        cos, sin = ang.cos(), ang.sin()
        x = self.embed_tokens(idx)
        for layer in self.layers:
            x = layer(x, cos, sin)
        logits = self.lm_head(self.norm(x))
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().view(-1, logits.size(-1)), targets.reshape(-1))


class PlainViT(nn.Module):
    """ViT-B/16 by default: 224 x 224 x 3 images, 16 x 16 patches + class token, 12 pre-LN blocks of width 768
    with 12 heads and MLP 3072, 1000 classes (non-causal attention)."""

    def __init__(self, image_size: int = 224, patch: int = 16, dim: int = 768, depth: int = 12, heads: int = 12,
                 num_classes: int = 1000) -> None:
        super().__init__()
        tokens = (image_size // patch) ** 2 + 1
        self.patch_embed = nn.Conv2d(3, dim, patch, stride=patch)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, dim))
        self.pos_embed = nn.Parameter(torch.randn(1, tokens, dim) * 0.02)
        self.blocks = nn.ModuleList([_Block(dim, heads, causal=False, eps=1e-6) for _ in range(depth)])
        self.norm = nn.LayerNorm(dim, eps=1e-6)
        self.head = nn.Linear(dim, num_classes)
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.trunc_normal_(m.weight, std=0.02)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)

    def forward(self, images, labels=None):
        B = images.shape[0]
        x = self.patch_embed(images).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls_token.expand(B, -1, -1), x], dim=1) + self.pos_embed
        for blk in self.blocks:
            x = blk(x)
        logits = self.head(self.norm(x)[:, 0])
        if labels is None:
            return logits
        return F.cross_entropy(logits.float(), labels)
