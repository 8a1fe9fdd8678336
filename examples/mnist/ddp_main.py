"""The MNIST-shaped example as data parallel across processes.

(reference: examples/mnist/ddp_main.py:25-107)

    torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node 2 -m examples.mnist.ddp_main --steps 200

Uses NCCL when CUDA is available and gloo otherwise; the input stream is
sharded by rank and seeded with ``seed + rank``.
"""

from __future__ import annotations

import argparse
import datetime
import os

import torch
import torch.distributed as dist


def main(argv=None):
    from koochak_b200.loop import training_loop
    from koochak_b200.optim.build import build_optimizer

    from .main import SyntheticMNIST, build_model, step_fn, train_config

    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--out", default="runs/mnist_ddp")
    ap.add_argument("--seed", type=int, default=42)
    args = ap.parse_args(argv)
    backend = "nccl" if torch.cuda.is_available() else "gloo"
    if not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    rank = dist.get_rank()
    try:
        torch.manual_seed(args.seed)
        model = build_model()
        opt = build_optimizer(model, {"name": "adamw", "lr": 1e-3})
        cfg = train_config(args.steps, args.out, ddp=True, seed=args.seed + rank, warn_unsharded=False)
        if torch.cuda.is_available():
            cfg["device"] = f"cuda:{int(os.environ.get('LOCAL_RANK', 0))}"
        return training_loop(model=model, dataset=SyntheticMNIST(64, seed=args.seed + rank), step_fn=step_fn,
                             optimizer=opt, train_cfg=cfg)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
