"""Memory-bound and attention kernels on the GPT-2 124M step shapes.

Each case is timed with CUDA events after warm-up and reported with the
bytes it must move (and the resulting bandwidth) or, for attention, its
FLOPs. The attention cases are also timed on PyTorch's SDPA (the library
attention on this GPU) for reference.

    python -m koochak_b200.benchmarks.kernels                  # all cases
    python -m koochak_b200.benchmarks.kernels --case norm_bwd
"""

from __future__ import annotations

import argparse
from typing import Callable, Dict, List, Tuple

import torch

from .gemm import time_ms

M, C, H, S, B, V = 16384, 768, 12, 1024, 16, 50304


def cases() -> Dict[str, Tuple[Callable[[], object], float, str]]:
    from koochak_b200.ops import functional as kf

    dev = "cuda"
    x = torch.randn(M, C, device=dev)
    w = torch.rand(C, device=dev) + 0.5
    bias = torch.randn(C, device=dev)
    dy16 = torch.randn(M, C, device=dev).bfloat16()
    dres = torch.randn(M, C, device=dev)
    _, mean, rstd = kf.norm_forward(x, w, bias, 1e-5, rms=False, out_dtype=torch.bfloat16)
    out: Dict[str, Tuple[Callable[[], object], float, str]] = {}
    out["norm_fwd"] = (lambda: kf.norm_forward(x, w, bias, 1e-5, rms=False, out_dtype=torch.bfloat16),
                       M * C * (4 + 2) + M * 8, "bytes")
    out["norm_bwd"] = (lambda: kf.norm_backward(dy16, x, w, mean, rstd, rms=False, dres=dres, dx_dtype=torch.float32,
                                                want_lp=True),
                       M * C * (2 + 4 + 4 + 4 + 2) + M * 8, "bytes")
    x2 = torch.randn(8192, 2048, device=dev)
    w2 = torch.rand(2048, device=dev) + 0.5
    dy2 = torch.randn(8192, 2048, device=dev).bfloat16()
    dr2 = torch.randn(8192, 2048, device=dev)
    _, _, r2 = kf.norm_forward(x2, w2, None, 1e-5, rms=True, out_dtype=torch.bfloat16)
    out["rmsnorm_bwd_2048"] = (lambda: kf.norm_backward(dy2, x2, w2, None, r2, rms=True, dres=dr2,
                                                        dx_dtype=torch.float32, want_lp=True),
                               8192 * 2048 * (2 + 4 + 4 + 4 + 2) + 8192 * 4, "bytes")
    g3072 = torch.randn(M, 3072, device=dev).bfloat16()
    out["bias_grad_3072"] = (lambda: kf.bias_grad(g3072), M * 3072 * 2, "bytes")
    logits = torch.randn(M, V, device=dev).bfloat16()
    tgt = torch.randint(0, 50257, (M,), device=dev)
    out["ce_fwd"] = (lambda: kf.cross_entropy_forward(logits, tgt, 50257), M * V * 2, "bytes")
    _, lse = kf.cross_entropy_forward(logits, tgt, 50257)
    gscale = torch.ones(1, device=dev)
    lg2 = logits.clone()
    out["ce_bwd"] = (lambda: kf.cross_entropy_backward_(lg2, tgt, lse, gscale, 50257), M * V * 4, "bytes")
    qkv = torch.randn(B, S, 3, H, 64, device=dev).bfloat16()
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    o, lse_a = kf.flash_attention_forward(q, k, v, causal=True)
    do = torch.randn_like(o)
    fl_fwd = 4.0 * B * H * S * S * 64 / 2  # causal
    sd = torch.nn.functional.scaled_dot_product_attention
    out["attn_fwd"] = (lambda: kf.flash_attention_forward(q, k, v, causal=True), fl_fwd, "flop")
    from koochak_b200.ops import native

    def fwd_mma_sync():
        native().attention_set_impl(1)
        try:
            return kf.flash_attention_forward(q, k, v, causal=True)
        finally:
            native().attention_set_impl(0)

    out["attn_fwd_mma_sync"] = (fwd_mma_sync, fl_fwd, "flop")
    qkv2 = torch.randn(4, 4096, 3, 16, 128, device=dev).bfloat16()
    q2, k2, v2 = qkv2[:, :, 0], qkv2[:, :, 1], qkv2[:, :, 2]
    fl2 = 4.0 * 4 * 16 * 4096 * 4096 * 128
    out["attn_fwd_d128_s4096"] = (lambda: kf.flash_attention_forward(q2, k2, v2, causal=False), fl2, "flop")
    q2t, k2t, v2t = (t.transpose(1, 2).contiguous() for t in (q2, k2, v2))

    def sdpa_fwd2():
        with torch.no_grad():
            return sd(q2t, k2t, v2t)

    out["attn_fwd_d128_s4096_sdpa"] = (sdpa_fwd2, fl2, "flop")
    out["attn_bwd"] = (lambda: kf.flash_attention_backward(q, k, v, o, do, lse_a, causal=True), 2.5 * fl_fwd, "flop")
    qt, kt, vt = (t.transpose(1, 2).contiguous().requires_grad_(True) for t in (q, k, v))

    def sdpa_fwd():
        with torch.no_grad():
            return sd(qt, kt, vt, is_causal=True)

    ot = sd(qt, kt, vt, is_causal=True)
    gt = torch.randn_like(ot)
    out["attn_fwd_sdpa"] = (sdpa_fwd, fl_fwd, "flop")
    out["attn_bwd_sdpa"] = (lambda: torch.autograd.grad(ot, (qt, kt, vt), gt, retain_graph=True), 2.5 * fl_fwd,
                            "flop")
    # Llama-style 1.3B: B4, H16, S2048, D128, causal.
    qkvl = torch.randn(4, 2048, 3, 16, 128, device=dev).bfloat16()
    ql, kl, vl = qkvl[:, :, 0], qkvl[:, :, 1], qkvl[:, :, 2]
    ol, lsel = kf.flash_attention_forward(ql, kl, vl, causal=True)
    dol = torch.randn_like(ol)
    fl_l = 4.0 * 4 * 16 * 2048 * 2048 * 128 / 2
    out["attn_fwd_llama"] = (lambda: kf.flash_attention_forward(ql, kl, vl, causal=True), fl_l, "flop")
    out["attn_bwd_llama"] = (lambda: kf.flash_attention_backward(ql, kl, vl, ol, dol, lsel, causal=True),
                             2.5 * fl_l, "flop")
    qlt, klt, vlt = (t.transpose(1, 2).contiguous().requires_grad_(True) for t in (ql, kl, vl))

    def sdpa_fwd_l():
        with torch.no_grad():
            return sd(qlt, klt, vlt, is_causal=True)

    olt = sd(qlt, klt, vlt, is_causal=True)
    glt = torch.randn_like(olt)
    out["attn_fwd_llama_sdpa"] = (sdpa_fwd_l, fl_l, "flop")
    out["attn_bwd_llama_sdpa"] = (lambda: torch.autograd.grad(olt, (qlt, klt, vlt), glt, retain_graph=True),
                                  2.5 * fl_l, "flop")
    return out


def main(argv: List[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--case", default="all")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    torch.manual_seed(0)
    for name, (fn, amount, kind) in cases().items():
        if args.case != "all" and not name.startswith(args.case):
            continue
        t = time_ms(fn, args.iters)
        rate = amount / (t * 1e-3)
        unit = f"{rate / 1e9:8.0f} GB/s" if kind == "bytes" else f"{rate / 1e12:8.0f} TF/s"
        print(f"{name:18s} {t * 1e3:9.1f} us  {unit}", flush=True)


if __name__ == "__main__":
    main()
