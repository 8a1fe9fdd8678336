"""Headline benchmark: GPT-2 124M training throughput (tokens/s) with Muon + AdamW, EMA and clipping.

Usage (one node, one process per GPU):

    python bench.py --gpus 1 --steps 20 --warmup 5
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W
    python bench.py --impl reference ...     # the reference framework on the same workload

Workload (per GPU, weak scaling): GPT-2 small (12 layers, d=768, 12 heads,
vocab 50257, seq 1024, tied LM head), micro-batch 16 x 1024 tokens, bf16
autocast, Muon (5 Newton-Schulz steps) on the hidden matrices and AdamW on
embeddings/norms/biases, EMA decay 0.999 (GPU-resident), gradient clip 1.0,
data parallel over all ranks. Synthetic uniform-random token ids,
random-init weights.

Timing: W untimed warm-up steps, then exactly K steps bracketed by a barrier
and ``torch.cuda.synchronize()`` on both sides, measured with CUDA events on
the training stream (device time), max over ranks. The step's working set
(about 6 GB of activations) is far larger than the 126 MB L2, so nothing
stays cache-resident between steps. A second phase ("e2e") runs the same
steps through the same public API with every step's batch copied from pinned
host memory and the loss read back to the host.

Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from typing import Any, Dict, List, Optional, Tuple

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "tokens/sec at 1/2/4/8 B200 (GPT-2 124M DDP+Muon); exposed comm ms/step"
BASELINE_VALUE: Optional[float] = None  # the reference publishes no throughput number


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["koochak_b200", "reference"], default="koochak_b200")
    ap.add_argument("--model", choices=["gpt2", "llama"], default="gpt2",
                    help="gpt2: GPT-2 124M (the headline workload); llama: Llama-style 1.3B, micro-batch 4 x 2048, "
                         "grad_accum 4")
    ap.add_argument("--micro-batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--grad-accum", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--bucket-mb", type=int, default=None,
                    help="data-parallel gradient bucket size in MB (train.ddp_bucket_cap_mb; both arms)")
    ap.add_argument("--comm", default="fused", help="gradient-sync transport: fused (in-kernel NVLink) | nccl")
    args = ap.parse_args()
    defaults = {"gpt2": dict(micro_batch=16, seq=1024, layers=12, grad_accum=1, vocab=50257),
                "llama": dict(micro_batch=4, seq=2048, layers=24, grad_accum=4, vocab=32000)}[args.model]
    for k, v in defaults.items():
        if getattr(args, k, None) is None:
            setattr(args, k, v)
    return args


# --------------------------------------------------------------------------- clocks


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu_index = gpu_index
        self.proc: Optional[subprocess.Popen] = None
        self.lines: List[Tuple[float, str]] = []  # (arrival time, csv line)
        self._thread: Optional[threading.Thread] = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return

        def read():
            assert self.proc is not None and self.proc.stdout is not None
            for line in self.proc.stdout:
                self.lines.append((time.perf_counter(), line.strip()))

        self._thread = threading.Thread(target=read, daemon=True)
        self._thread.start()

    def stop(self, t_lo: Optional[float] = None, t_hi: Optional[float] = None) -> Dict[str, Any]:
        """Stop sampling; summarise the samples that arrived in [t_lo, t_hi].

        The sampler is started during warm-up, so a timed region shorter than
        the sampling period still has samples under load: when none arrived
        inside the window, the ones from the second before it are used and
        ``window`` says so.
        """

        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        window = "timed"
        picked = [ln for t, ln in self.lines if (t_lo is None or t >= t_lo) and (t_hi is None or t <= t_hi)]
        if not picked and t_lo is not None:
            picked = [ln for t, ln in self.lines if t_lo - 1.0 <= t <= (t_hi if t_hi is not None else t_lo)]
            window = "last second of warm-up"
        for line in picked:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "window": window}


# --------------------------------------------------------------------------- workloads


def build_koochak_workload(args, device):
    import torch

    from koochak_b200.models import GPT2
    from koochak_b200.optim import build_optimizer

    torch.manual_seed(1234)
    if args.model == "llama":
        from koochak_b200.models import Llama

        model = Llama(n_layer=args.layers, max_seq_len=args.seq).to(device)
    else:
        model = GPT2(n_layer=args.layers).to(device)
    opt = build_optimizer(model, {"name": "muon", "lr": 6e-4, "muon_lr": 0.02, "adam_lr": 6e-4,
                                  "weight_decay": 0.0})
    return model, opt


def step_fn(model, batch, ctx):
    return {"loss": model(batch["idx"], batch["targets"])}


def synthetic_batches(n: int, micro: int, seq: int, vocab: int, device, pinned: bool, seed: int):
    import torch

    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        tok = torch.randint(0, vocab, (micro, seq + 1), generator=g)
        b = {"idx": tok[:, :-1].contiguous(), "targets": tok[:, 1:].contiguous()}
        if pinned:
            b = {k: v.pin_memory() for k, v in b.items()}
        else:
            b = {k: v.to(device) for k, v in b.items()}
        out.append(b)
    return out


class CyclingDataset:
    """Yields a fixed pool of batches in order, forever (fresh dict per step)."""

    def __init__(self, pool):
        self.pool = pool

    def __iter__(self):
        i = 0
        while True:
            yield dict(self.pool[i % len(self.pool)])
            i += 1


def train_cfg_for(args, world: int, steps: int, out_dir: str, scalarize: bool) -> Dict[str, Any]:
    return {
        "max_steps": steps, "log_every": 10 ** 9, "eval_every": 0, "ckpt_every": 10 ** 9,
        "grad_clip_norm": 1.0, "amp": "bf16", "ddp": world > 1, "out_dir": out_dir, "keep_last_k": 1,
        "scalarize_loss_every_step": scalarize, "ema": {"enabled": True, "decay": 0.999, "offload_to_cpu": False},
        "comm_transport": args.comm, "warn_unsharded": False, "grad_accum": args.grad_accum,
        **({"ddp_bucket_cap_mb": args.bucket_mb} if args.bucket_mb else {}),
    }


class StepTimer:
    """on_update_end hook: device events around steps [warmup, warmup+steps), bracketed by barriers."""

    def __init__(self, warmup: int, steps: int, world: int, sampler: Optional[ClockSampler], wall: bool,
                 native_counter=None):
        import torch

        self.warmup, self.steps, self.world = warmup, steps, world
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)
        self.sampler = sampler
        self.wall = wall
        self.t0 = self.t1 = 0.0
        self.native_counter = native_counter
        self.launch0 = self.launch1 = 0
        self.clocks: Optional[Dict[str, Any]] = None

    def _barrier(self):
        import torch

        torch.cuda.synchronize()
        if self.world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def __call__(self, log, ctx):
        step = int(ctx["step"])
        if step == 0 and self.warmup > 1 and self.sampler is not None:
            self.sampler.start()  # during warm-up: nvidia-smi needs a few hundred ms for its first sample
        if step == self.warmup - 1:
            self._barrier()
            if self.sampler is not None and self.sampler.proc is None:
                self.sampler.start()
            if self.native_counter is not None:
                self.launch0 = self.native_counter()
            self.t0 = time.perf_counter()
            self.start.record()
        elif step == self.warmup + self.steps - 1:
            self.end.record()
            self._barrier()
            self.t1 = time.perf_counter()
            if self.native_counter is not None:
                self.launch1 = self.native_counter()
            if self.sampler is not None:
                self.clocks = self.sampler.stop(self.t0, self.t1)

    def ms_per_step(self) -> float:
        if self.wall:
            return (self.t1 - self.t0) * 1000.0 / self.steps
        return self.start.elapsed_time(self.end) / self.steps


def max_over_ranks(value: float, world: int) -> float:
    import torch

    if world <= 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


class NoGradSyncHook:
    """on_update_end hook that turns the data-parallel gradient sync off from the first update on.

    Used to time the same step without gradient communication: the
    difference to the normal step is the communication left exposed.
    """

    def __call__(self, log, ctx):
        model = ctx.get("model")
        if model is None:
            return
        if hasattr(model, "require_sync"):
            model.require_sync = False  # koochak_b200 DataParallel
        if hasattr(model, "require_backward_grad_sync"):
            model.require_backward_grad_sync = False  # torch DistributedDataParallel


def run_phase(impl: str, args, world: int, rank: int, device, *, e2e: bool, sampler=None,
              no_grad_sync: bool = False) -> Dict[str, Any]:
    import torch

    total = args.warmup + args.steps
    if impl == "koochak_b200":
        from koochak_b200.loop import training_loop
        from koochak_b200.ops import native

        model, opt = build_koochak_workload(args, device)
        counter = native().launch_count
    else:
        training_loop, model, opt = build_reference_workload(args, device)
        counter = None
    pool = synthetic_batches(4, args.micro_batch, args.seq, args.vocab, device, pinned=e2e, seed=100 + rank)
    timer = StepTimer(args.warmup, args.steps, world, sampler, wall=e2e, native_counter=counter)
    with tempfile.TemporaryDirectory(prefix="kb_bench_") as out_dir:
        cfg = train_cfg_for(args, world, total, out_dir, scalarize=e2e)
        hooks = [NoGradSyncHook(), timer] if no_grad_sync else [timer]
        training_loop(model=model, dataset=CyclingDataset(pool), step_fn=step_fn, optimizer=opt, train_cfg=cfg,
                      hooks={"on_update_end": hooks})
    ms = max_over_ranks(timer.ms_per_step(), world)
    h2d = sum(v.numel() * v.element_size() for v in pool[0].values()) if e2e else 0
    return {"ms_per_step": ms, "clocks": timer.clocks, "launches": timer.launch1 - timer.launch0,
            "h2d": h2d, "d2h": 4 if e2e else 0}


# --------------------------------------------------------------------------- reference arm


def build_reference_workload(args, device):
    """The reference framework, installed unmodified under baseline/_ref, on a plain-PyTorch GPT-2."""

    ref_root = os.path.join(HERE, "baseline", "_ref")
    shim = os.path.join(HERE, "baseline", "shims")
    if not os.path.isdir(os.path.join(ref_root, "koochak")):
        raise RuntimeError("reference not installed under baseline/_ref")
    for p in (ref_root, shim):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch

    from koochak.loop import training_loop  # type: ignore
    from koochak.optim import build as ref_build  # type: ignore
    from koochak.utils.nn_utils import tag_param  # type: ignore

    sys.path.insert(0, os.path.join(HERE, "baseline"))
    from reference_workloads import PlainGPT2, PlainLlama  # type: ignore

    torch.manual_seed(1234)
    if args.model == "llama":
        model = PlainLlama(n_layer=args.layers).to(device)
        mats = model.blocks_matrices()
    else:
        model = PlainGPT2(n_layer=args.layers).to(device)
        mats = [w for blk in model.blocks for w in blk.matrices()]
    for w in mats:
        tag_param(w, "wd")
    opt = ref_build.build_optimizer(model, {"name": "muon", "lr": 6e-4, "muon_lr": 0.02, "adam_lr": 6e-4,
                                            "weight_decay": 0.0})
    return training_loop, model, opt


# --------------------------------------------------------------------------- main


def main() -> int:
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and not os.path.isdir(os.path.join(HERE, "baseline", "_ref", "koochak")):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}))
        return 0
    import datetime

    import torch

    if args.warmup < 1 or args.steps < 1:
        raise SystemExit("--warmup and --steps must be >= 1")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=device)
    sampler = ClockSampler(local) if rank == 0 else None
    res = run_phase(args.impl, args, world, rank, device, e2e=False, sampler=sampler)
    tokens_per_step = args.micro_batch * args.seq * args.grad_accum * world
    value = tokens_per_step / (res["ms_per_step"] / 1000.0)
    e2e = None
    if not args.no_e2e:
        r2 = run_phase(args.impl, args, world, rank, device, e2e=True)
        e2e = {"value": tokens_per_step / (r2["ms_per_step"] / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": r2["h2d"], "d2h_bytes_per_step": r2["d2h"], "ms_per_step": r2["ms_per_step"]}
    exposed = 0.0 if world == 1 else None
    if world > 1:
        r3 = run_phase(args.impl, args, world, rank, device, e2e=False, no_grad_sync=True)
        exposed = max(0.0, res["ms_per_step"] - r3["ms_per_step"])
    out = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None, "dtype": "bf16",
        "data": "synthetic uniform-random token ids, random-init weights",
        "config": {"model": (f"GPT-2 124M ({args.layers}L, d768, 12 heads, vocab 50257, tied head)"
                             if args.model == "gpt2" else
                             f"Llama-style 1.3B ({args.layers}L, d2048, 16 heads, RMSNorm, RoPE, SwiGLU 5504, "
                             "vocab 32000)"),
                   "global_batch": args.micro_batch * args.grad_accum * world,
                   "micro_batch_per_gpu": args.micro_batch, "grad_accum": args.grad_accum,
                   "seq_len": args.seq, "parallelism": f"dp{world}", "optimizer": "Muon(NS5)+AdamW",
                   "ema_decay": 0.999, "grad_clip": 1.0,
                   "l2": "no flush: per-step working set (~6 GB activations) >> 126 MB L2"},
        "clocks": res["clocks"], "e2e": e2e,
    }
    # Exposed gradient-sync time: this step minus the same step with the
    # data-parallel gradient sync switched off (device-timed, max over ranks).
    out["exposed_comm_ms"] = exposed
    if args.impl == "reference":
        out["impl"] = "reference"
    else:
        out["gpu_launches"] = res["launches"]
        out["comm_transport"] = args.comm
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
