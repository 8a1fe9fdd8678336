"""Data parallel on CPU with gloo, two ranks: the MNIST-shaped MLP workload.

* ranks end with identical parameters (gradients were averaged);
* a run stopped at step 10 resumes from its checkpoint and finishes at
  step 20 with ranks still identical (checkpoint save / resume round trip);
* the CLI trains the example config end to end.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out: str, steps: int, resume: str) -> None:
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from examples.mnist.main import SyntheticMNIST, build_model, step_fn, train_config
        from koochak_b200.loop import training_loop
        from koochak_b200.optim.build import build_optimizer

        torch.manual_seed(42)
        model = build_model()
        opt = build_optimizer(model, {"name": "adamw", "lr": 1e-3})
        cfg = train_config(steps, os.path.join(out, "ckpt"), ddp=True, seed=42 + rank, warn_unsharded=False,
                           ckpt_every=10, log_every=1000)
        training_loop(model=model, dataset=SyntheticMNIST(64, seed=42 + rank), step_fn=step_fn, optimizer=opt,
                      train_cfg=cfg, resume=resume)
        torch.save({k: v.detach().clone() for k, v in model.state_dict().items()},
                   os.path.join(out, f"final_rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _run(out, steps, resume="none"):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _port(), str(out), steps, resume), nprocs=2, join=True)
    return [torch.load(os.path.join(out, f"final_rank{r}.pt")) for r in range(2)]


def test_ddp_two_ranks_identical_and_resume(tmp_path):
    full = _run(tmp_path / "full", 20)
    for k in full[0]:
        torch.testing.assert_close(full[0][k], full[1][k], rtol=0, atol=0)
    _run(tmp_path / "part", 10)
    # Resume from the step-10 checkpoint and continue to step 20.
    resumed = _run(tmp_path / "part", 20, resume="auto")
    for k in full[0]:
        torch.testing.assert_close(resumed[0][k], resumed[1][k], rtol=0, atol=0)
    ck = sorted(p for p in os.listdir(tmp_path / "part" / "ckpt") if p.endswith(".pt") and p.startswith("step"))
    assert ck[-1] == "step000000020.pt"
    state = torch.load(tmp_path / "part" / "ckpt" / ck[-1], weights_only=False)
    assert state["next_step"] == 20 and "optimizer" in state and "rng" in state


def test_cli_trains_example(tmp_path):
    from koochak_b200.cli.train import main

    cfg = tmp_path / "run.yaml"
    text = open(os.path.join(os.path.dirname(__file__), "..", "examples", "mnist", "config.yaml")).read()
    cfg.write_text(text.replace("max_steps: 200", "max_steps: 12").replace("eval_every: 100", "eval_every: 6")
                   .replace("ckpt_every: 100", "ckpt_every: 6").replace("./runs/mnist_cli", str(tmp_path / "out")))
    main(["--config", str(cfg), "--resume", "none"])
    names = os.listdir(tmp_path / "out")
    assert "step000000012.pt" in names and "step000000012.pt.ready.json" in names and "log.jsonl" in names
