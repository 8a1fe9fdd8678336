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
    def __init__(self, d: int, h: int) -> None:
        super().__init__()
        self.h = h
        self.c_attn = nn.Linear(d, 3 * d)
        self.c_proj = nn.Linear(d, d)

    def forward(self, x):
        B, S, C = x.shape
        q, k, v = self.c_attn(x).view(B, S, 3, self.h, C // self.h).unbind(2)
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        return self.c_proj(y.transpose(1, 2).reshape(B, S, C))


class _Block(nn.Module):
    def __init__(self, d: int, h: int) -> None:
        super().__init__()
        self.ln_1 = nn.LayerNorm(d)
        self.attn = _Attn(d, h)
        self.ln_2 = nn.LayerNorm(d)
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
