"""GEMM benchmark: the native tcgen05 GEMM against cuBLAS on the model shapes.

Shapes are the linear layers of GPT-2 124M at 16 x 1024 tokens per GPU
(M = 16384; d = 768, FFN 3072, vocab 50304 padded) and the Newton-Schulz
GEMMs of Muon on 12 stacked 768 x c matrices. Each case is timed with CUDA
events after warm-up; the inputs of the linear cases stay resident in L2
(this measures the kernels, not DRAM).

    python -m koochak_b200.benchmarks.gemm                 # every case
    python -m koochak_b200.benchmarks.gemm --case fc --op fwd --iters 4 --no-compare
"""

from __future__ import annotations

import argparse
from typing import Callable, Dict, List, Tuple

import torch

LINEAR: Dict[str, Tuple[int, int]] = {  # name -> (N out, K in)
    "qkv": (2304, 768),
    "attn_proj": (768, 768),
    "fc": (3072, 768),
    "mlp_proj": (768, 3072),
    "lm_head": (50304, 768),
}

# Llama-style 1.3B at 4 x 2048 tokens per GPU (M = 8192): fused q/k/v, output
# projection, fused gate/up, down projection, LM head.
LINEAR_LLAMA: Dict[str, Tuple[int, int]] = {
    "l_qkv": (6144, 2048),
    "l_o": (2048, 2048),
    "l_gate_up": (11008, 2048),
    "l_down": (2048, 5504),
    "l_lm_head": (32000, 2048),
}


def time_ms(fn: Callable[[], object], iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def linear_cases(name: str, M: int, block_n: int):
    from koochak_b200.ops import functional as kf

    N, K = LINEAR[name]
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    dy = torch.randn(M, N, device="cuda").bfloat16()
    flops = 2.0 * M * N * K
    return flops, {
        "fwd": (lambda: kf.gemm(x, w, block_n=block_n), lambda: torch.matmul(x, w.t())),
        "dgrad": (lambda: kf.gemm(dy, w, b_mn_major=True, block_n=block_n), lambda: torch.matmul(dy, w)),
        "wgrad": (lambda: kf.gemm(dy, x, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32, block_n=block_n),
                  lambda: torch.matmul(dy.t(), x)),
    }


def ns_cases(c: int, batch: int = 12, r: int = 768, block_n: int = 0):
    from koochak_b200.ops import functional as kf

    X = torch.randn(batch, r, c, device="cuda").bfloat16()
    A = torch.randn(batch, r, r, device="cuda").bfloat16()
    return {
        "XXt": (2.0 * batch * r * r * c, lambda: kf.gemm(X, X, block_n=block_n),
                lambda: torch.bmm(X, X.transpose(1, 2))),
        "XXt_sym": (2.0 * batch * r * r * c, lambda: kf.gemm(X, X, block_n=block_n, symmetric=True),
                    lambda: torch.bmm(X, X.transpose(1, 2))),
        "AA": (2.0 * batch * r ** 3, lambda: kf.gemm(A, A, d=A, alpha=2.0, beta=-4.0, block_n=block_n),
               lambda: torch.bmm(A, A)),
        "AA_sym": (2.0 * batch * r ** 3, lambda: kf.gemm(A, A, d=A, alpha=2.0, beta=-4.0, block_n=block_n,
                                                          symmetric=True),
                   lambda: torch.bmm(A, A)),
        "BX": (2.0 * batch * r * r * c, lambda: kf.gemm(A, X, b_mn_major=True, d=X, beta=3.0, block_n=block_n),
               lambda: torch.bmm(A, X)),
    }


def wait_profile(fn: Callable[[], object]) -> str:
    """Fractions of the producer role's time that each role spent waiting, for one launch."""

    from koochak_b200.ops import native

    buf = torch.zeros(4096, dtype=torch.int64, device="cuda")
    native().gemm_set_profile(buf)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        native().gemm_set_profile(None)
    c = buf.view(-1, 8).double()
    active = c[:, 4] > 0
    c = c[active]
    total = c[:, 4].sum().clamp_min(1)
    return ("wait: load-slot {:.0%} mma-operands {:.0%} mma-accum {:.0%} epi-accum/warp {:.0%} "
            "tiles/cta {:.1f}").format(float(c[:, 0].sum() / total), float(c[:, 1].sum() / total),
                                      float(c[:, 2].sum() / total), float(c[:, 3].sum() / 8 / total),
                                      float(c[:, 5].sum() / max(1, int((c[:, 5] > 0).sum()))))


def main(argv: List[str] | None = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--case", default="all", help="linear layer name, 'ns<c>' (e.g. ns768) or 'all'")
    ap.add_argument("--op", default="all", help="fwd | dgrad | wgrad | XXt | XXt_sym | AA | AA_sym | BX | all")
    ap.add_argument("--tokens", type=int, default=None, help="M (default 16384 for gpt2, 8192 for llama)")
    ap.add_argument("--model", choices=["gpt2", "llama"], default="gpt2",
                    help="which model's linear and Newton-Schulz shapes 'all' covers")
    ap.add_argument("--block-n", type=int, default=0, help="0 auto; 128/256 one-SM tiles; -128/-256 two-SM tiles")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-compare", action="store_true", help="skip the cuBLAS comparison")
    ap.add_argument("--shape", default=None, help="M,N,K: one extra forward case of that shape (name 'custom')")
    ap.add_argument("--debug-mode", type=int, default=0,
                    help="diagnostic GEMM mode for timing studies: 1 skips operand loads, 2 skips the epilogue")
    ap.add_argument("--group", type=int, default=-1,
                    help="tile-column group width of the tile order (-1: the built-in rule; 0/1: plain order)")
    ap.add_argument("--split", type=int, default=-1,
                    help="K-cut of fp32 outputs: -1 the built-in rule, 0 none, 1 stream-K, s >= 2 split-K")
    ap.add_argument("--profile", action="store_true",
                    help="also report where each role of the GEMM waited (clock64 counters per CTA)")
    args = ap.parse_args(argv)
    torch.manual_seed(0)
    if args.tokens is None:
        args.tokens = 16384 if args.model == "gpt2" else 8192
    LINEAR.update(LINEAR_LLAMA)
    if args.shape:
        m, n, k = (int(v) for v in args.shape.split(","))
        LINEAR["custom"] = (n, k)
        args.tokens = m
    if args.group >= 0:
        from koochak_b200.ops import native

        native().gemm_set_group(args.group)
    if args.split >= 0:
        from koochak_b200.ops import native

        native().gemm_set_split(args.split)
    if args.debug_mode:
        from koochak_b200.ops import native

        native().gemm_set_debug(args.debug_mode)
    if args.case != "all":
        names = [args.case]
    elif args.model == "gpt2":
        names = [n for n in LINEAR if n not in LINEAR_LLAMA] + ["ns768", "ns2304", "ns3072"]
    else:
        names = list(LINEAR_LLAMA) + ["nsL2048", "nsL5504"]
    for name in names:
        if name.startswith("nsL"):
            # Llama Muon batches: 2048 x c matrices, 8 per batch (one rank's share at 8 GPUs x 3)
            cases = ns_cases(int(name[3:]), batch=8, r=2048, block_n=args.block_n)
            items = [(op, fl, a, b) for op, (fl, a, b) in cases.items()]
        elif name.startswith("ns"):
            cases = ns_cases(int(name[2:]), block_n=args.block_n)
            items = [(op, fl, a, b) for op, (fl, a, b) in cases.items()]
        else:
            fl, cases = linear_cases(name, args.tokens, args.block_n)
            items = [(op, fl, a, b) for op, (a, b) in cases.items()]
        for op, fl, ours, ref in items:
            if args.op != "all" and op != args.op:
                continue
            t = time_ms(ours, args.iters)
            line = f"{name:10s} {op:6s} ours {t * 1e3:8.1f} us {fl / t / 1e9:6.0f} TF/s"
            if args.profile:
                line += " | " + wait_profile(ours)
            if not args.no_compare:
                tr = time_ms(ref, args.iters)
                line += f" | cublas {tr * 1e3:8.1f} us {fl / tr / 1e9:6.0f} TF/s | ratio {tr / t:.2f}"
            print(line, flush=True)


if __name__ == "__main__":
    main()
