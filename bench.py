"""Headline benchmark: GPT-2 124M training throughput (tokens/s) with Muon + AdamW, EMA and clipping.

Usage (one node, one process per GPU):

    python bench.py --gpus 1 --steps 40 --warmup 5
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

``--model vit`` runs ViT-B/16 (224 x 224 x 3 images drawn i.i.d. N(0,1),
1000 classes with uniform labels, batch 128 per GPU) under fp16 autocast with
the dynamic GradScaler, AdamW at lr 1e-3 with a cosine schedule and EMA
0.999. Every 100 updates (at update 10, 110, ...) the step's loss is
multiplied by 1e30 so the fp16 backward overflows. Two variants:
``--vit-clip none`` (no clipping: the overflowing update is skipped by the
scaler; the line reports how many updates the optimizer actually ran) and
``--vit-clip 1.0`` (clip 1.0: the clip raises ``FloatingPointError`` on the
non-finite gradients; the overflow is forced on the first update after the
timed ones and the line reports the exception). Metric: images/s.

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
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["koochak_b200", "reference"], default="koochak_b200")
    ap.add_argument("--model", choices=["gpt2", "llama", "vit"], default="gpt2",
                    help="gpt2: GPT-2 124M (the headline workload); llama: Llama-style 1.3B, micro-batch 4 x 2048, "
                         "grad_accum 4; vit: ViT-B/16, batch 128, fp16 + GradScaler with forced overflow")
    ap.add_argument("--vit-clip", choices=["none", "1.0"], default="none",
                    help="ViT only: none = overflowing updates are skipped; 1.0 = clip 1.0, the overflow raises")
    ap.add_argument("--overflow-every", type=int, default=100, help="ViT only: forced-overflow period in updates")
    ap.add_argument("--micro-batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--grad-accum", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--bucket-mb", type=int, default=None,
                    help="data-parallel gradient bucket size in MB (train.ddp_bucket_cap_mb; both arms)")
    ap.add_argument("--comm", default="fused", help="gradient-sync transport: fused (in-kernel NVLink) | nccl")
    ap.add_argument("--no-graph", action="store_true",
                    help="run forward + backward eagerly (no CUDA-graph capture of the single-GPU step)")
    args = ap.parse_args()
    defaults = {"gpt2": dict(micro_batch=16, seq=1024, layers=12, grad_accum=1, vocab=50257),
                "llama": dict(micro_batch=4, seq=2048, layers=24, grad_accum=4, vocab=32000),
                "vit": dict(micro_batch=128, seq=197, layers=12, grad_accum=1, vocab=1000)}[args.model]
    for k, v in defaults.items():
        if getattr(args, k, None) is None:
            setattr(args, k, v)
    return args


# --------------------------------------------------------------------------- clocks


class ClockSampler:
    """Samples SM clocks, power and throttle reasons of one GPU while the timed region runs.

    NVML is polled every 50 ms on a thread (read-only queries), so even a
    timed region of half a second holds about ten samples; where NVML cannot
    be loaded, ``nvidia-smi -lms 200`` is read instead. The GPU is found by
    its PCI bus id, so the index order of CUDA and NVML need not agree.
    """

    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.05

    def __init__(self, cuda_index: int) -> None:
        self.cuda_index = cuda_index
        self.samples: List[Tuple[float, float, float, frozenset]] = []  # (time, sm MHz, max MHz, reasons)
        self.source = "none"
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._proc: Optional[subprocess.Popen] = None

    @property
    def running(self) -> bool:
        return self._thread is not None

    def _nvml_poller(self):
        import pynvml  # nvidia-ml-py

        import torch

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.cuda_index)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        masks = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
        smax = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))

        def poll():
            try:
                while not self._stop.is_set():
                    sm = float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                    bits = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle))
                    active = frozenset(n for n, m in masks.items() if bits & m)
                    self.samples.append((time.perf_counter(), sm, smax, active))
                    self._stop.wait(self.PERIOD_S)
            finally:
                pynvml.nvmlShutdown()

        return poll

    def _smi_poller(self):
        self._proc = subprocess.Popen(["nvidia-smi", "-i", str(self.cuda_index), f"--query-gpu={self.SMI_FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)

        def read():
            assert self._proc is not None and self._proc.stdout is not None
            for line in self._proc.stdout:
                parts = [p.strip() for p in line.split(",")]
                try:
                    sm, smax = float(parts[1]), float(parts[2])
                except (ValueError, IndexError):
                    continue
                active = frozenset(n for n, v in zip(self.REASONS, parts[5:9]) if v.lower() == "active")
                self.samples.append((time.perf_counter(), sm, smax, active))

        return read

    def start(self) -> None:
        try:
            target, self.source = self._nvml_poller(), "nvml"
        except Exception:  # NVML missing or the bus id unknown: fall back to nvidia-smi
            try:
                target, self.source = self._smi_poller(), "nvidia-smi"
            except OSError:
                self.source = "none"
                return
        self._thread = threading.Thread(target=target, daemon=True)
        self._thread.start()

    def stop(self, t_lo: Optional[float] = None, t_hi: Optional[float] = None) -> Dict[str, Any]:
        """Stop sampling; summarise the samples taken in [t_lo, t_hi].

        The sampler is started during warm-up, so a timed region shorter than
        the sampling period still has samples under load: when none fall
        inside the window, the ones from the second before it are used and
        ``window`` says so.
        """

        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=2)
        window = "timed"
        picked = [x for x in self.samples if (t_lo is None or x[0] >= t_lo) and (t_hi is None or x[0] <= t_hi)]
        if not picked and t_lo is not None:
            picked = [x for x in self.samples if t_lo - 1.0 <= x[0] <= (t_hi if t_hi is not None else t_lo)]
            window = "last second of warm-up"
        sm = [x[1] for x in picked]
        reasons = sorted(set().union(*[x[3] for x in picked])) if picked else []
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": picked[-1][2] if picked else None,
                "reasons": reasons, "samples": len(sm), "window": window, "source": self.source}


# --------------------------------------------------------------------------- workloads


def build_koochak_workload(args, device):
    import torch

    from koochak_b200.models import GPT2
    from koochak_b200.optim import build_optimizer, build_scheduler

    torch.manual_seed(1234)
    if args.model == "vit":
        from koochak_b200.models import ViT

        model = ViT(depth=args.layers).to(device)
        opt = build_optimizer(model, VIT_OPTIM)
        return model, opt, build_scheduler(opt, VIT_SCHED, {"max_steps": args.warmup + args.steps})
    if args.model == "llama":
        from koochak_b200.models import Llama

        model = Llama(n_layer=args.layers, max_seq_len=args.seq).to(device)
    else:
        model = GPT2(n_layer=args.layers).to(device)
    return model, build_optimizer(model, MUON_OPTIM), None


MUON_OPTIM = {"name": "muon", "lr": 6e-4, "muon_lr": 0.02, "adam_lr": 6e-4, "weight_decay": 0.0}
VIT_OPTIM = {"name": "adamw", "lr": 1e-3, "weight_decay": 0.05}
VIT_SCHED = {"name": "cosine"}
OVERFLOW_PHASE = 10


def step_fn(model, batch, ctx):
    return {"loss": model(batch["idx"], batch["targets"])}


class VitStep:
    """step_fn for the ViT workload: mean cross-entropy times a device scalar, 1 or 1e30.

    The scalar is 1e30 on the forced-overflow updates (the fp16 backward then
    overflows and the scaler sees inf gradients). It lives on the device and is
    set by ``advance`` (an ``on_update_end`` hook) for the next update, so the
    step_fn computes the same thing on every update and the step can be
    replayed from a CUDA graph.
    """

    def __init__(self, overflow_at):
        self.overflow_at = overflow_at  # step -> bool
        self.mult = None

    def _ensure(self, device):
        import torch

        if self.mult is None:
            self.mult = torch.full((), 1e30 if self.overflow_at(0) else 1.0, device=device)

    def __call__(self, model, batch, ctx):
        self._ensure(batch["images"].device)
        return {"loss": model(batch["images"], batch["labels"]) * self.mult}

    def advance(self, log, ctx):
        """on_update_end: the multiplier of update ctx['step'] + 1."""

        if self.mult is not None:
            self.mult.fill_(1e30 if self.overflow_at(int(ctx["step"]) + 1) else 1.0)


def vit_batches(n: int, micro: int, device, pinned: bool, seed: int):
    import torch

    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        b = {"images": torch.randn((micro, 3, 224, 224), generator=g),
             "labels": torch.randint(0, 1000, (micro,), generator=g)}
        b = {k: (v.pin_memory() if pinned else v.to(device)) for k, v in b.items()}
        out.append(b)
    return out


class OptimizerStepCounter:
    """on_update_end hook: how many updates ran and how many the optimizer applied (its ``step`` state)."""

    def __init__(self, optimizer):
        self.param = next(p for g in optimizer.param_groups for p in g["params"])
        self.optimizer = optimizer
        self.updates = 0

    def __call__(self, log, ctx):
        self.updates += 1

    def applied(self) -> int:
        st = self.optimizer.state.get(self.param, {})
        return int(st.get("step", 0))


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


def train_cfg_for(args, world: int, steps: int, out_dir: str, scalarize: bool, impl: str) -> Dict[str, Any]:
    vit = args.model == "vit"
    clip = (None if args.vit_clip == "none" else float(args.vit_clip)) if vit else 1.0
    # This framework's loop captures forward + backward as one CUDA graph on a single GPU with one
    # micro-batch per update (GPT-2 and ViT; the Llama step accumulates four micro-batches and stays eager).
    # The capture happens during warm-up, so every timed update replays it.
    graph = (impl == "koochak_b200" and not args.no_graph)
    return {
        **({"cuda_graph_step": True, "cuda_graph_warmup": max(1, args.warmup - 2)} if graph else {}),
        "max_steps": steps, "log_every": 10 ** 9, "eval_every": 0, "ckpt_every": 10 ** 9,
        "grad_clip_norm": clip, "amp": "fp16" if vit else "bf16", "ddp": world > 1, "out_dir": out_dir,
        "keep_last_k": 1,
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
            self.sampler.start()  # during warm-up: the first samples take a moment to arrive
        if step == self.warmup - 1:
            self._barrier()
            if self.sampler is not None and not self.sampler.running:
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
    total = args.warmup + args.steps
    if impl == "koochak_b200":
        from koochak_b200.loop import training_loop
        from koochak_b200.ops import native

        model, opt, sched = build_koochak_workload(args, device)
        counter = native().launch_count
    else:
        training_loop, model, opt, sched = build_reference_workload(args, device)
        counter = None
    vit = args.model == "vit"
    raise_variant = vit and args.vit_clip != "none"
    if vit:
        pool = vit_batches(2, args.micro_batch, device, pinned=e2e, seed=100 + rank)
        if raise_variant:  # one overflowing update right after the timed ones
            fn = VitStep(lambda step: step == total)
        else:
            every = max(1, args.overflow_every)
            fn = VitStep(lambda step: step % every == OVERFLOW_PHASE % every)
    else:
        pool = synthetic_batches(4, args.micro_batch, args.seq, args.vocab, device, pinned=e2e, seed=100 + rank)
        fn = step_fn
    timer = StepTimer(args.warmup, args.steps, world, sampler, wall=e2e, native_counter=counter)
    steps_counter = OptimizerStepCounter(opt)
    outcome = "completed"
    with tempfile.TemporaryDirectory(prefix="kb_bench_") as out_dir:
        cfg = train_cfg_for(args, world, total + (1 if raise_variant else 0), out_dir, scalarize=e2e, impl=impl)
        hooks = ([NoGradSyncHook()] if no_grad_sync else []) + [timer, steps_counter]
        if isinstance(fn, VitStep):
            hooks.append(fn.advance)
        try:
            training_loop(model=model, dataset=CyclingDataset(pool), step_fn=fn, optimizer=opt, scheduler=sched,
                          train_cfg=cfg, hooks={"on_update_end": hooks})
        except FloatingPointError:
            if not raise_variant:
                raise
            outcome = "FloatingPointError"
    ms = max_over_ranks(timer.ms_per_step(), world)
    h2d = sum(v.numel() * v.element_size() for v in pool[0].values()) if e2e else 0
    return {"ms_per_step": ms, "clocks": timer.clocks, "launches": timer.launch1 - timer.launch0,
            "h2d": h2d, "d2h": 4 if e2e else 0, "outcome": outcome, "updates": steps_counter.updates,
            "optimizer_steps": steps_counter.applied()}


# --------------------------------------------------------------------------- reference arm


def build_reference_workload(args, device):
    """The reference framework, installed unmodified under baseline/_ref, on a plain-PyTorch model of the workload."""

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
    from reference_workloads import PlainGPT2, PlainLlama, PlainViT  # type: ignore

    torch.manual_seed(1234)
    if args.model == "vit":
        model = PlainViT(depth=args.layers).to(device)
        opt = ref_build.build_optimizer(model, VIT_OPTIM)
        sched = ref_build.build_scheduler(opt, VIT_SCHED, {"max_steps": args.warmup + args.steps})
        return training_loop, model, opt, sched
    if args.model == "llama":
        model = PlainLlama(n_layer=args.layers).to(device)
        mats = model.blocks_matrices()
    else:
        model = PlainGPT2(n_layer=args.layers).to(device)
        mats = [w for blk in model.blocks for w in blk.matrices()]
    for w in mats:
        tag_param(w, "wd")
    return training_loop, model, ref_build.build_optimizer(model, MUON_OPTIM), None


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
    vit = args.model == "vit"
    samples_per_step = args.micro_batch * args.grad_accum * world
    per_step = samples_per_step if vit else samples_per_step * args.seq
    unit = "images/s" if vit else "tokens/s"
    value = per_step / (res["ms_per_step"] / 1000.0)
    e2e = None
    if not args.no_e2e:
        r2 = run_phase(args.impl, args, world, rank, device, e2e=True)
        e2e = {"value": per_step / (r2["ms_per_step"] / 1000.0), "unit": unit,
               "h2d_bytes_per_step": r2["h2d"], "d2h_bytes_per_step": r2["d2h"], "ms_per_step": r2["ms_per_step"]}
    exposed = 0.0 if world == 1 else None
    if world > 1:
        r3 = run_phase(args.impl, args, world, rank, device, e2e=False, no_grad_sync=True)
        exposed = max(0.0, res["ms_per_step"] - r3["ms_per_step"])
    if vit:
        model_desc = f"ViT-B/16 ({args.layers}L, d768, 12 heads, MLP 3072, 224x224x3, 197 tokens, 1000 classes)"
        data = "synthetic images i.i.d. N(0,1) and uniform labels, random-init weights"
        optim = "AdamW lr 1e-3, wd 0.05, cosine schedule"
        clip = None if args.vit_clip == "none" else float(args.vit_clip)
        l2 = "no flush: per-step working set (~20 GB activations) >> 126 MB L2"
    else:
        model_desc = (f"GPT-2 124M ({args.layers}L, d768, 12 heads, vocab 50257, tied head)" if args.model == "gpt2"
                      else f"Llama-style 1.3B ({args.layers}L, d2048, 16 heads, RMSNorm, RoPE, SwiGLU 5504, "
                           "vocab 32000)")
        data = "synthetic uniform-random token ids, random-init weights"
        optim = "Muon(NS5)+AdamW"
        clip = 1.0
        l2 = "no flush: per-step working set (~6 GB activations) >> 126 MB L2"
    out = {
        "metric": METRIC if args.model == "gpt2" else f"{unit} ({args.model})", "value": value, "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE and args.model == "gpt2" else None,
        "dtype": "fp16" if vit else "bf16", "data": data,
        "config": {"model": model_desc, "global_batch": samples_per_step,
                   "micro_batch_per_gpu": args.micro_batch, "grad_accum": args.grad_accum,
                   "seq_len": args.seq, "parallelism": f"dp{world}", "optimizer": optim,
                   "ema_decay": 0.999, "grad_clip": clip, "l2": l2,
                   "fwd_bwd_cuda_graph": bool(args.impl == "koochak_b200" and not args.no_graph
                                              and world == 1 and args.grad_accum == 1)},
        "clocks": res["clocks"], "e2e": e2e,
    }
    if vit:
        # Forced overflow: without clipping the scaler skips the update (optimizer steps < updates run);
        # with clipping the non-finite gradients raise.
        out["overflow"] = {"every": args.overflow_every, "phase": OVERFLOW_PHASE,
                           "variant": "skip" if clip is None else "raise",
                           "updates_run": res["updates"], "optimizer_steps": res["optimizer_steps"],
                           "outcome": res["outcome"]}
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
