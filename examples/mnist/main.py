"""MNIST-shaped MLP trained through ``training_loop`` on synthetic data.

(the usage example of reference examples/mnist/main.py, reshaped to the
784 -> 256 ReLU -> 10 classifier the benchmarks use)

    python -m examples.mnist.main --steps 200 --out runs/mnist
    python -m koochak_b200.cli.train --config examples/mnist/config.yaml

Images are uniform in [0, 1) of shape 1 x 28 x 28 and labels uniform over
0..9, drawn from a fixed seed, so the example needs no download.
"""

from __future__ import annotations

import argparse
from typing import Dict, Iterator

import torch
import torch.nn as nn
import torch.nn.functional as F


class MLP(nn.Module):
    def __init__(self, hidden: int = 256) -> None:
        super().__init__()
        self.fc1 = nn.Linear(28 * 28, hidden)
        self.fc2 = nn.Linear(hidden, 10)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(F.relu(self.fc1(x.flatten(1))))


class SyntheticMNIST(torch.utils.data.IterableDataset):
    """Endless batches of (image, label); ``seed`` fixes the stream."""

    def __init__(self, batch_size: int = 64, seed: int = 0, length: int | None = None) -> None:
        self.batch_size, self.seed, self.length = batch_size, seed, length

    def __iter__(self) -> Iterator[Dict[str, torch.Tensor]]:
        g = torch.Generator().manual_seed(self.seed)
        i = 0
        while self.length is None or i < self.length:
            yield {"x": torch.rand(self.batch_size, 1, 28, 28, generator=g),
                   "y": torch.randint(0, 10, (self.batch_size,), generator=g)}
            i += 1


def build_model() -> nn.Module:
    return MLP()


def build_dataset():
    return SyntheticMNIST(batch_size=64, seed=0)


def build_eval_dataset():
    return SyntheticMNIST(batch_size=256, seed=1, length=4)


def step_fn(model, batch, ctx):
    logits = model(batch["x"])
    loss = F.cross_entropy(logits, batch["y"])
    return {"loss": loss, "acc": (logits.argmax(-1) == batch["y"]).float().mean().detach()}


@torch.no_grad()
def eval_fn(model, dataset, ctx):
    tot, n = 0.0, 0
    for batch in dataset:
        batch = {k: v.to(ctx.get("device", "cpu")) for k, v in batch.items()}
        tot += float(F.cross_entropy(model(batch["x"]), batch["y"], reduction="sum"))
        n += batch["y"].numel()
    return {"val_loss": tot / max(n, 1)}


def train_config(steps: int, out_dir: str, **extra) -> Dict:
    cfg = {"max_steps": steps, "log_every": 50, "eval_every": 0, "ckpt_every": steps, "grad_clip_norm": 1.0,
           "amp": "fp32", "out_dir": out_dir, "keep_last_k": 2,
           "ema": {"enabled": True, "decay": 0.999, "offload_to_cpu": False}}
    cfg.update(extra)
    return cfg


def main(argv=None) -> Dict:
    from koochak_b200.loop import training_loop
    from koochak_b200.logging import make_stdout_hooks
    from koochak_b200.optim.build import build_optimizer

    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--out", default="runs/mnist")
    args = ap.parse_args(argv)
    torch.manual_seed(42)
    model = build_model()
    opt = build_optimizer(model, {"name": "adamw", "lr": 1e-3})
    return training_loop(model=model, dataset=build_dataset(), step_fn=step_fn, optimizer=opt,
                         train_cfg=train_config(args.steps, args.out), eval_dataset=build_eval_dataset(),
                         eval_fn=eval_fn, hooks=make_stdout_hooks())


if __name__ == "__main__":
    main()
