"""Where a training step's time goes: kernel time in place, and the GPU's idle gaps with their causes.

Runs the benchmark workloads (GPT-2 124M, Llama-style 1.3B, ViT-B/16 with
the same shapes, optimizer, EMA and clipping as ``bench.py``) through
``training_loop`` on one GPU and records ``--steps`` updates after
``--warmup`` with ``torch.profiler`` (CUPTI activity records of kernels and
CUDA runtime calls). It then reports

* the window, the time some kernel was running (intervals of all streams
  merged) and the idle rest;
* every idle gap longer than ``--gap-us``, attributed to the CUDA runtime
  call the host was inside when the GPU ran dry (a synchronisation, an
  allocation, a copy) or, when there is none, to host-side launch latency;
* each kernel's time as it ran in the step (warm caches, real clocks), which
  a kernel profiler's serialised replay does not give.

The profiler's own host overhead (a few microseconds per launch) lengthens
launch-bound gaps somewhat; the causes it names stay valid.

    python -m koochak_b200.benchmarks.timeline --model llama --steps 2 --warmup 3 --out timeline.txt
"""

from __future__ import annotations

import argparse
import collections
import os
import sys
import tempfile
from typing import Any, Dict, List, Tuple

import torch

_SYNC_CALLS = ("cudaStreamSynchronize", "cudaDeviceSynchronize", "cudaEventSynchronize", "cudaMemcpy",
               "cudaMalloc", "cudaFree", "cudaHostAlloc", "cudaMemset", "cudaStreamWaitEvent", "cuMemcpy",
               "cudaMemcpyAsync")


def _workload(model: str, device):
    from koochak_b200.models import GPT2, Llama, ViT
    from koochak_b200.optim import build_optimizer, build_scheduler

    torch.manual_seed(1234)
    g = torch.Generator().manual_seed(7)
    if model == "vit":
        net = ViT().to(device)
        opt = build_optimizer(net, {"name": "adamw", "lr": 1e-3, "weight_decay": 0.05})
        batch = {"images": torch.randn((128, 3, 224, 224), generator=g).to(device),
                 "labels": torch.randint(0, 1000, (128,), generator=g).to(device)}

        def step_fn(m, b, ctx):
            return {"loss": m(b["images"], b["labels"])}

        cfg = {"amp": "fp16", "grad_clip_norm": None}
        return net, opt, build_scheduler(opt, {"name": "cosine"}, {"max_steps": 1000}), batch, step_fn, cfg
    if model == "llama":
        net = Llama(n_layer=24, max_seq_len=2048).to(device)
        micro, seq, vocab, accum = 4, 2048, 32000, 4
    else:
        net = GPT2(n_layer=12).to(device)
        micro, seq, vocab, accum = 16, 1024, 50257, 1
    opt = build_optimizer(net, {"name": "muon", "lr": 6e-4, "muon_lr": 0.02, "adam_lr": 6e-4, "weight_decay": 0.0})
    tok = torch.randint(0, vocab, (micro, seq + 1), generator=g)
    batch = {"idx": tok[:, :-1].contiguous().to(device), "targets": tok[:, 1:].contiguous().to(device)}

    def step_fn(m, b, ctx):
        return {"loss": m(b["idx"], b["targets"])}

    return net, opt, None, batch, step_fn, {"amp": "bf16", "grad_clip_norm": 1.0, "grad_accum": accum}


def _merge(intervals: List[Tuple[float, float]]) -> List[Tuple[float, float]]:
    out: List[Tuple[float, float]] = []
    for s, e in sorted(intervals):
        if out and s <= out[-1][1]:
            out[-1] = (out[-1][0], max(out[-1][1], e))
        else:
            out.append((s, e))
    return out


def analyse(events, gap_us: float) -> Dict[str, Any]:
    """Kernel busy time, idle gaps with causes, and per-kernel totals from profiler events (times in us)."""

    kernels, runtime, ops = [], [], []
    for e in events:
        dev = str(getattr(e, "device_type", ""))
        start, end = float(e.time_range.start), float(e.time_range.end)
        if dev.endswith("CUDA"):
            if not getattr(e, "is_user_annotation", False) and "#" not in e.name:
                kernels.append((start, end, e.name))
        elif e.name.startswith(("cuda", "cu")):
            runtime.append((start, end, e.name))
        else:
            ops.append((start, end, e.name, tuple(getattr(e, "stack", None) or ())))
    if not kernels:
        return {"error": "no kernel events recorded"}
    kernels.sort()
    busy = _merge([(s, e) for s, e, _ in kernels])
    t0, t1 = busy[0][0], busy[-1][1]
    busy_us = sum(e - s for s, e in busy)
    gaps = []
    for (s0, e0), (s1, e1) in zip(busy, busy[1:]):
        if s1 - e0 >= gap_us:
            gaps.append((e0, s1))
    runtime.sort()
    causes: Dict[str, List[float]] = collections.defaultdict(lambda: [0, 0.0])
    stacks: Dict[str, set] = collections.defaultdict(set)
    gap_rows = []
    for gs, ge in gaps:
        # The runtime call that ended last before the GPU resumed and overlapped the gap the most.
        best, best_ov, best_call = "host launch latency", 0.0, None
        for rs, re_, name in runtime:
            if re_ < gs or rs > ge:
                continue
            ov = min(re_, ge) - max(rs, gs)
            if name.startswith(_SYNC_CALLS) and ov > best_ov:
                best, best_ov, best_call = name, ov, (rs, re_)
        if best_call is not None:
            # The host operators enclosing that call, innermost first (e.g. aten::item < gate code).
            rs, re_ = best_call
            enclosing = sorted((o for o in ops if o[0] <= rs and o[1] >= re_), key=lambda o: o[1] - o[0])
            names = [o[2] for o in enclosing if not o[2].startswith("ProfilerStep")][:3]
            if names:
                best = best + " in " + " < ".join(names)
            frames = next((o[3] for o in enclosing if o[3]), ())
            if frames:
                stacks[best].add(" <- ".join(f for f in frames[:6]))
        causes[best][0] += 1
        causes[best][1] += ge - gs
        before = max((k for k in kernels if k[1] <= gs + 0.5), key=lambda k: k[1], default=None)
        after = min((k for k in kernels if k[0] >= ge - 0.5), key=lambda k: k[0], default=None)
        gap_rows.append((ge - gs, best, before[2] if before else "-", after[2] if after else "-"))
    # Host operators running while the GPU was idle (nested operators each count their own overlap).
    host_in_gaps: Dict[str, float] = collections.defaultdict(float)
    ops.sort()
    for gs, ge in gaps:
        for os_, oe, name, _stack in ops:
            if os_ >= ge:
                break
            if oe > gs:
                host_in_gaps[name] += min(oe, ge) - max(os_, gs)
    # Host time of the loop's named phases (the loop.* ranges): where the host spends each step.
    host_phases: Dict[str, float] = collections.defaultdict(float)
    for os_, oe, name, _stack in ops:
        if name.startswith("loop."):
            host_phases[name] += oe - os_
    per_kernel: Dict[str, List[float]] = collections.defaultdict(lambda: [0, 0.0])
    for s, e, name in kernels:
        per_kernel[name][0] += 1
        per_kernel[name][1] += e - s
    return {"window_us": t1 - t0, "busy_us": busy_us, "idle_us": (t1 - t0) - busy_us, "n_kernels": len(kernels),
            "causes": dict(causes), "gaps": sorted(gap_rows, reverse=True), "per_kernel": dict(per_kernel),
            "host_in_gaps": dict(host_in_gaps), "stacks": {k: sorted(v) for k, v in stacks.items()},
            "host_phases": dict(host_phases)}


def report(res: Dict[str, Any], steps: int, top: int = 40) -> str:
    if "error" in res:
        return res["error"]
    lines = []
    w, b, i = res["window_us"] / 1e3, res["busy_us"] / 1e3, res["idle_us"] / 1e3
    lines.append(f"window {w:.2f} ms over {steps} step(s): kernels running {b:.2f} ms ({100 * b / w:.1f}%), "
                 f"idle {i:.2f} ms; {res['n_kernels']} kernels")
    lines.append(f"per step: window {w / steps:.2f} ms, busy {b / steps:.2f} ms, idle {i / steps:.2f} ms")
    lines.append("")
    lines.append("idle gaps by cause (count, total ms):")
    for name, (n, us) in sorted(res["causes"].items(), key=lambda x: -x[1][1]):
        lines.append(f"  {us / 1e3:9.3f} ms  {int(n):6d}  {name[:150]}")
    lines.append("")
    lines.append(f"largest gaps (us, cause, kernel before -> kernel after):")
    for us, cause, before, after in res["gaps"][:top]:
        lines.append(f"  {us:9.1f}  {cause[:90]:90s} {before[:50]} -> {after[:50]}")
    lines.append("")
    if res.get("host_phases"):
        lines.append("host time of the loop's phases per step (ms):")
        for name, us in sorted(res["host_phases"].items(), key=lambda x: -x[1]):
            lines.append(f"  {us / 1e3 / steps:9.3f} ms  {name}")
        lines.append("")
    if res.get("stacks"):
        lines.append("Python stacks of the synchronising calls (innermost frame first):")
        for cause, frames in res["stacks"].items():
            lines.append(f"  {cause[:100]}")
            for f in frames[:4]:
                lines.append(f"      {f[:300]}")
        lines.append("")
    lines.append("host operators running during those gaps (ms of overlap; nested operators each counted):")
    for name, us in sorted(res.get("host_in_gaps", {}).items(), key=lambda x: -x[1])[:top]:
        lines.append(f"  {us / 1e3:9.3f} ms  {name[:120]}")
    lines.append("")
    lines.append("kernels as they ran (total ms, launches, share of busy time):")
    for name, (n, us) in sorted(res["per_kernel"].items(), key=lambda x: -x[1][1])[:top]:
        lines.append(f"  {us / 1e3:9.3f} ms {int(n):6d} {100 * us / res['busy_us']:5.1f}%  {name[:110]}")
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", choices=["gpt2", "llama", "vit"], default="gpt2")
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--gap-us", type=float, default=10.0)
    ap.add_argument("--out", default=None)
    ap.add_argument("--stacks", action="store_true", help="record Python stacks (slower host) to locate syncs")
    ap.add_argument("--graph", action="store_true",
                    help="capture forward + backward as a CUDA graph (train.cuda_graph_step; one micro-batch)")
    args = ap.parse_args(argv)
    from torch.profiler import ProfilerActivity, profile

    from koochak_b200.loop import training_loop

    os.environ.setdefault("KAVEH_PROFILE_RANGES", "1")  # the optimizer's named host ranges

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    model, opt, sched, batch, step_fn, extra = _workload(args.model, device)
    prof = profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], record_shapes=False,
                   with_stack=bool(args.stacks))
    first, last = args.warmup, args.warmup + args.steps - 1

    def hook(log, ctx):
        step = int(ctx["step"])
        if step == first - 1:
            torch.cuda.synchronize()
            prof.__enter__()
        elif step == last:
            torch.cuda.synchronize()
            prof.__exit__(None, None, None)

    def data():
        while True:
            yield dict(batch)

    cfg = {"max_steps": last + 1, "log_every": 10 ** 9, "eval_every": 0, "ckpt_every": 10 ** 9, "keep_last_k": 1,
           "scalarize_loss_every_step": False,  # as in bench.py's device-timed phase
           "ema": {"enabled": True, "decay": 0.999, "offload_to_cpu": False}, "warn_unsharded": False, **extra}
    if args.graph:
        cfg.update(cuda_graph_step=True, cuda_graph_warmup=max(1, args.warmup - 2))
    with tempfile.TemporaryDirectory(prefix="kb_timeline_") as out_dir:
        cfg["out_dir"] = out_dir
        training_loop(model=model, dataset=data(), step_fn=step_fn, optimizer=opt, scheduler=sched, train_cfg=cfg,
                      hooks={"on_update_end": [hook]})
    text = report(analyse(prof.events(), args.gap_us), args.steps)
    text = f"model {args.model}, steps {args.steps} after {args.warmup} warm-up\n" + text
    print(text)
    if args.out:
        os.makedirs(os.path.dirname(os.path.abspath(args.out)), exist_ok=True)
        with open(args.out, "w") as f:
            f.write(text + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
