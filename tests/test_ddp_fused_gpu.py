"""Data parallel with the fused NVLink gradient sync and the sharded optimizer, end to end on 2 GPUs.

Two ranks train a small GPT-2 through ``training_loop`` (``ddp: true``,
``comm_transport: fused``): Muon matrices reduced into their owner only
(matrix i of the size-sorted group on rank i % 2), every Adam tensor
reduce-scattered and updated sharded, new parameters stored into both
ranks' copies from inside the update kernels. The oracle is one GPU training
the same model on the concatenated batch (the same tokens, so the same mean
gradient up to summation order). After 5 steps:

* both ranks hold bit-identical parameters;
* every parameter's distance from the one-GPU result is small against the
  distance the training moved it (bf16 autocast and a different reduction
  order keep them from being bitwise equal);
* the checkpoint written at step 5 carries every Muon matrix's momentum and
  the complete Adam moments (gathered from the owners), close to the one-GPU
  optimizer state.
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


STEPS = 5
MICRO = 4
SEQ = 256
VOCAB = 4096


def _batches(rank_count: int, rank: int):
    """Step s's batch of this rank: rows [rank*MICRO, (rank+1)*MICRO) of the global batch of step s."""

    out = []
    for s in range(STEPS):
        g = torch.Generator().manual_seed(500 + s)
        tok = torch.randint(0, VOCAB, (2 * MICRO, SEQ + 1), generator=g)
        rows = tok if rank_count == 1 else tok[rank * MICRO:(rank + 1) * MICRO]
        out.append({"idx": rows[:, :-1].contiguous(), "targets": rows[:, 1:].contiguous()})
    return out


class _Data:
    def __init__(self, pool):
        self.pool = pool

    def __iter__(self):
        i = 0
        while True:
            yield dict(self.pool[i % len(self.pool)])
            i += 1


def _step_fn(model, batch, ctx):
    return {"loss": model(batch["idx"], batch["targets"])}


def _train(rank: int, world: int, out: str) -> None:
    from koochak_b200.loop import training_loop
    from koochak_b200.models import GPT2
    from koochak_b200.optim import build_optimizer

    dev = torch.device("cuda", rank)
    torch.manual_seed(0)
    model = GPT2(n_layer=2, n_head=4, n_embd=256, vocab_size=VOCAB, block_size=SEQ).to(dev)
    init = {k: v.detach().clone().cpu() for k, v in model.state_dict().items()}
    opt = build_optimizer(model, {"name": "muon", "lr": 3e-3, "muon_lr": 0.02, "adam_lr": 3e-3, "weight_decay": 0.0})
    pool = [{k: v.to(dev) for k, v in b.items()} for b in _batches(world, rank)]
    cfg = {"max_steps": STEPS, "log_every": 10 ** 9, "eval_every": 0, "ckpt_every": STEPS, "grad_clip_norm": 1.0,
           "amp": "bf16", "ddp": world > 1, "out_dir": os.path.join(out, f"ck{world}"), "keep_last_k": 2,
           "comm_transport": "fused", "warn_unsharded": False, "scalarize_loss_every_step": False}
    training_loop(model=model, dataset=_Data(pool), step_fn=_step_fn, optimizer=opt, train_cfg=cfg)
    torch.cuda.synchronize()
    final = {k: v.detach().clone().cpu() for k, v in model.state_dict().items()}
    torch.save({"init": init, "final": final}, os.path.join(out, f"params_w{world}_r{rank}.pt"))


def _worker(rank: int, world: int, port: int, out: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), KOOCHAK_B200_COMM_TIMEOUT_S="30")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=90),
                            device_id=torch.device("cuda", rank))
    try:
        _train(rank, world, out)
    finally:
        dist.destroy_process_group()


def _single(out: str) -> None:
    _train(0, 1, out)


@pytest.mark.gpu
def test_fused_ddp_sharded_optimizer_matches_one_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_single, args=(str(tmp_path),))
    p.start()
    p.join()
    assert p.exitcode == 0
    r0 = torch.load(tmp_path / "params_w2_r0.pt")
    r1 = torch.load(tmp_path / "params_w2_r1.pt")
    one = torch.load(tmp_path / "params_w1_r0.pt")
    for k, v in r0["final"].items():
        assert torch.equal(v, r1["final"][k]), f"ranks differ on {k}"
        moved = float((one["final"][k] - one["init"][k]).abs().max())
        diff = float((v - one["final"][k]).abs().max())
        assert diff <= 0.1 * moved + 1e-6, f"{k}: |2 GPUs - 1 GPU| = {diff:.3g}, training moved it {moved:.3g}"
    c2 = torch.load(tmp_path / "ck2" / f"step{STEPS:09d}.pt", weights_only=False)["optimizer"]["state"]
    c1 = torch.load(tmp_path / "ck1" / f"step{STEPS:09d}.pt", weights_only=False)["optimizer"]["state"]
    assert set(c2) == set(c1), "gathered checkpoint does not hold the same optimizer entries as one GPU"
    for i, st in c1.items():
        for key, ref in st.items():
            if not torch.is_tensor(ref):
                assert c2[i][key] == ref
                continue
            got = c2[i][key].float()
            scale = float(ref.float().abs().max()) + 1e-12
            assert float((got - ref.float()).abs().max()) <= 0.15 * scale, f"state {i} {key} differs"
