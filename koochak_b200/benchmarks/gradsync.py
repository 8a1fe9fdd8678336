"""Gradient-sync and optimizer-step microbenchmark (one node, 2-8 GPUs).

Workload: a synthetic parameter set of fp32 matrices and vectors with the
GPT-2 124M shapes (``--preset gpt2``: 12 x [2304x768, 768x768, 3072x768,
768x3072] + embeddings/norm/bias vectors, 124M values) or the Llama-style
1.3B ones (``--preset llama``), gradients drawn N(0, 1e-3). Phases, each timed
with CUDA events on the launching stream after warm-up, max over ranks:

* ``sync``: gradient reduction + GradScaler unscale + finite flag +
  per-tensor sums of squares + clip coefficient.
  - fused: one kernel per bucket (``--bucket-mb``, default 25) over NVLink
    (``FusedGradReducer``, P2P or NVSwitch multimem), then the seal + gate
    kernel. Two plans: ``allreduce`` (every reduced value to every rank) and
    ``sharded`` (what the sharded optimizer asks for: matrix i of the
    size-sorted Muon group reduced into rank i % W only, every vector
    reduce-scattered);
  - nccl: ``dist.all_reduce`` per bucket, then the unscale/finite/norm pass
    (``torch._amp_foreach_non_finite_check_and_unscale_`` + per-tensor
    ``torch._foreach_norm``), i.e. what torch DDP + GradScaler + clipping do.
* ``muon``: the sharded Muon step of the matrices (momentum, Newton-Schulz 5
  on tcgen05, update) followed by the parameter all-gather:
  - peer: the update kernel stores every owned matrix into all ranks' copies
    (symmetric slab, P2P or multimem) + one bounded barrier;
  - nccl: the same update, then one NCCL all-gather per shape bucket.

Roofline for ``sync``: the bytes that must cross NVLink per GPU per
direction, at the measured 770 GB/s: 2 (W-1)/W B for an all-reduce of B
bytes, (W-1)/W B for the sharded plan (each element reduced once, by one rank).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m koochak_b200.benchmarks.gradsync --preset gpt2

With one process (``RANK=0 WORLD_SIZE=1 MASTER_ADDR=127.0.0.1 MASTER_PORT=<p>
python -m koochak_b200.benchmarks.gradsync``) the same kernels run with every
peer access landing on the local GPU: the case a kernel profiler can capture.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
from typing import Dict, List, Tuple

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured peer copy bandwidth per direction per GPU


def shapes(preset: str) -> Tuple[List[Tuple[int, int]], List[int]]:
    if preset == "gpt2":
        d, L, V = 768, 12, 50304
        mats = [(3 * d, d), (d, d), (4 * d, d), (d, 4 * d)] * L
        vecs = [V * d, 1024 * d] + [d] * (L * 9 + 2) + [3 * d, 4 * d] * L
        return mats, vecs
    if preset == "llama":
        d, L, F, V = 2048, 24, 5504, 32000
        mats = [(d, d)] * 4 * L + [(F, d), (F, d), (d, F)] * L
        vecs = [V * d, V * d] + [d] * (2 * L + 1)
        return mats, vecs
    raise ValueError(preset)


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def bench_sync(grads: List[torch.Tensor], n_mats: int, iters: int, warmup: int, blocks: List[int],
               bucket_mb: float) -> Dict[str, float]:
    from koochak_b200.parallel.ddp import split_buckets
    from koochak_b200.parallel.symm import FusedGradReducer

    world = dist.get_world_size()
    sizes = [g.numel() for g in grads]
    # Gradient order: reverse of registration, as backward produces them.
    order = list(reversed(range(len(grads))))
    buckets = [[order[j] for j in b] for b in split_buckets([sizes[i] for i in order], [int(bucket_mb * 2 ** 20 / 4)])]
    segs = [[(sizes[i], i) for i in b] for b in buckets]
    scale = torch.tensor([1024.0], device="cuda")
    # Muon ownership: matrix i of the size-sorted group on rank i % W.
    by_size = sorted(range(n_mats), key=lambda i: sizes[i], reverse=True)
    owners = {t: k % world for k, t in enumerate(by_size)}
    out: Dict[str, float] = {"buckets": float(len(buckets))}
    nbytes = 4 * sum(sizes)
    for plan, owner_of, shard_rest in (("allreduce", {}, False), ("sharded", owners, True)):
        for nb in blocks:
            red = FusedGradReducer(segs, len(grads), grads[0].device, blocks=nb, owner_of=owner_of,
                                   shard_rest=shard_rest)
            for b in range(len(buckets)):
                for (off, n, t) in red.layouts[b]:
                    red.buffers[b][off:off + n].copy_(grads[t].view(-1))

            def fused():
                red.begin_step()
                for b in range(len(buckets)):
                    red.reduce(b, scale)
                red.seal_gate(1.0)

            out[f"{plan}_ms_blocks{nb}"] = _time(fused, iters, warmup)
            out["multimem"] = float(bool(red.ws.mc_base))
            del red
            torch.cuda.empty_cache()
        best = min(v for k, v in out.items() if k.startswith(f"{plan}_ms_blocks"))
        out[f"{plan}_ms"] = best
        mult = 2.0 if plan == "allreduce" else 1.0
        out[f"{plan}_roofline_ms"] = mult * (world - 1) / world * nbytes / (LINK_GBS * 1e9) * 1e3
        out[f"{plan}_frac_of_roofline"] = out[f"{plan}_roofline_ms"] / best

    flat = [torch.cat([grads[i].view(-1) for i in b]) for b in buckets]
    views = []
    for f, b in zip(flat, buckets):
        views += list(torch.split(f, [sizes[i] for i in b]))
    found = torch.zeros(1, device="cuda")
    inv = torch.tensor([1.0 / 1024.0], device="cuda")

    def nccl():
        for f in flat:
            dist.all_reduce(f)
            f.div_(world)
        torch._amp_foreach_non_finite_check_and_unscale_(views, found, inv)
        norms = torch.stack(torch._foreach_norm(views))
        total = torch.linalg.vector_norm(norms.double())
        torch.clamp(1.0 / (total + 1e-6), max=1.0)

    out.update({"nccl_ms": _time(nccl, iters, warmup), "grad_bytes": float(nbytes)})
    return out


def bench_muon(mats: List[Tuple[int, int]], iters: int, warmup: int, dev: torch.device) -> Dict[str, float]:
    from koochak_b200.optim.muon import MuonWithAuxAdam

    res = {}
    for mode in ("peer", "nccl"):
        os.environ["KOOCHAK_B200_MUON_GATHER"] = mode
        g = torch.Generator(device="cpu").manual_seed(0)
        params = [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).to(dev)) for s in mats]
        for p in params:
            p.grad = torch.randn_like(p) * 1e-3
        opt = MuonWithAuxAdam([dict(params=params, use_muon=True, lr=0.02, weight_decay=0.01)])
        if dist.get_world_size() == 1:
            # One process (a profiler capture): run the sharded code path with this rank owning everything.
            opt._distributed_now = lambda: True
        res[f"{mode}_ms"] = _time(opt.step, iters, warmup)
        del opt, params
        torch.cuda.empty_cache()
    os.environ.pop("KOOCHAK_B200_MUON_GATHER", None)
    res["param_bytes"] = float(4 * sum(r * c for r, c in mats))
    return res


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", choices=["gpt2", "llama"], default="gpt2")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--phase", choices=["sync", "muon", "all"], default="all")
    ap.add_argument("--blocks", default="32", help="comma-separated CTA counts of the fused reduction to time")
    ap.add_argument("--bucket-mb", type=float, default=25.0, help="gradient bucket size")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        mats, vecs = shapes(args.preset)
        out: Dict[str, object] = {"preset": args.preset, "world": dist.get_world_size(),
                                  "params": sum(r * c for r, c in mats) + sum(vecs)}
        if args.phase in ("sync", "all"):
            g = torch.Generator(device="cpu").manual_seed(1 + rank)
            grads = [(torch.randn(r * c, generator=g) * 1e-3).to(dev) for r, c in mats]
            grads += [(torch.randn(n, generator=g) * 1e-3).to(dev) for n in vecs]
            out["sync"] = bench_sync(grads, len(mats), args.iters, args.warmup,
                                     [int(b) for b in args.blocks.split(",")], args.bucket_mb)
            del grads
            torch.cuda.empty_cache()
        if args.phase in ("muon", "all"):
            out["muon"] = bench_muon(mats, args.iters, args.warmup, dev)
        if rank == 0:
            print(json.dumps(out))
    finally:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
