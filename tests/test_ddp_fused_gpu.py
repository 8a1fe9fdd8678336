"""Data parallel with the fused NVLink gradient sync and the sharded optimizer, end to end on 2 GPUs.

Two ranks train a small GPT-2 through ``training_loop`` (``ddp: true``,
``comm_transport: fused``): Muon matrices reduced into their owner only
(matrix i of the size-sorted group on rank i % 2), every Adam tensor
reduce-scattered and updated sharded, new parameters stored into both
ranks' copies from inside the update kernels.

Oracles:

* the same two ranks with ``comm_transport: nccl`` (torch-style all-reduce,
  replicated AdamW). With two ranks both paths average the same pair of
  values (a + b, then x 1/2: exact either way), so the gradients, and hence
  every update, must agree bit for bit; so must the gathered optimizer state
  in the step-5 checkpoint (every Muon momentum, full Adam moments);
* one GPU on the concatenated batch, for the Muon matrices only: its bf16
  products see a different batch split, so its gradients differ in the last
  bits. Muon's orthogonalised update is insensitive to that, AdamW with
  eps = 1e-10 is not (a near-zero gradient's sign decides a full lr step), so
  Adam tensors are checked against the NCCL run only.

Both ranks must also hold bit-identical parameters.
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


def _train(rank: int, world: int, out: str, transport: str = "fused") -> None:
    from koochak_b200.loop import training_loop
    from koochak_b200.models import GPT2
    from koochak_b200.optim import build_optimizer

    dev = torch.device("cuda", rank)
    torch.manual_seed(0)
    model = GPT2(n_layer=2, n_head=4, n_embd=256, vocab_size=VOCAB, block_size=SEQ).to(dev)
    init = {k: v.detach().clone().cpu() for k, v in model.state_dict().items()}
    opt = build_optimizer(model, {"name": "muon", "lr": 3e-3, "muon_lr": 0.02, "adam_lr": 3e-3, "weight_decay": 0.0})
    pool = [{k: v.to(dev) for k, v in b.items()} for b in _batches(world, rank)]
    cfg = {"max_steps": STEPS, "log_every": 10 ** 9, "eval_every": 0, "ckpt_every": STEPS, "grad_clip_norm": None,
           "amp": "bf16", "ddp": world > 1, "out_dir": os.path.join(out, f"ck{world}{transport}"), "keep_last_k": 2,
           "comm_transport": transport, "warn_unsharded": False, "scalarize_loss_every_step": False}
    training_loop(model=model, dataset=_Data(pool), step_fn=_step_fn, optimizer=opt, train_cfg=cfg)
    torch.cuda.synchronize()
    final = {k: v.detach().clone().cpu() for k, v in model.state_dict().items()}
    torch.save({"init": init, "final": final}, os.path.join(out, f"params_w{world}{transport}_r{rank}.pt"))


def _worker(rank: int, world: int, port: int, out: str, transport: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), KOOCHAK_B200_COMM_TIMEOUT_S="30")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=90),
                            device_id=torch.device("cuda", rank))
    try:
        _train(rank, world, out, transport)
    finally:
        dist.destroy_process_group()


def _single(out: str) -> None:
    _train(0, 1, out, "fused")


@pytest.mark.gpu
def test_fused_ddp_sharded_optimizer_matches_nccl_and_one_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    for transport in ("fused", "nccl"):
        mp.spawn(_worker, args=(2, _port(), str(tmp_path), transport), nprocs=2, join=True)
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_single, args=(str(tmp_path),))
    p.start()
    p.join()
    assert p.exitcode == 0
    fused = [torch.load(tmp_path / f"params_w2fused_r{r}.pt") for r in range(2)]
    nccl = torch.load(tmp_path / "params_w2nccl_r0.pt")
    one = torch.load(tmp_path / "params_w1fused_r0.pt")
    muon_like = [k for k, v in one["final"].items() if v.dim() == 2 and ".h." in k]
    assert muon_like, "no hidden matrices found"
    for k, v in fused[0]["final"].items():
        assert torch.equal(v, fused[1]["final"][k]), f"ranks differ on {k}"
        assert torch.equal(v, nccl["final"][k]), f"fused and NCCL runs differ on {k}: " \
            f"{float((v - nccl['final'][k]).abs().max()):.3g}"
    for k in muon_like:
        moved = float((one["final"][k] - one["init"][k]).abs().max())
        diff = float((fused[0]["final"][k] - one["final"][k]).abs().max())
        assert diff <= 0.1 * moved, f"{k}: |2 GPUs - 1 GPU| = {diff:.3g}, training moved it {moved:.3g}"
    c2 = torch.load(tmp_path / "ck2fused" / f"step{STEPS:09d}.pt", weights_only=False)["optimizer"]["state"]
    cn = torch.load(tmp_path / "ck2nccl" / f"step{STEPS:09d}.pt", weights_only=False)["optimizer"]["state"]
    c1 = torch.load(tmp_path / "ck1fused" / f"step{STEPS:09d}.pt", weights_only=False)["optimizer"]["state"]
    assert set(c2) == set(cn) == set(c1), "gathered checkpoints do not hold every optimizer entry"
    for i, st in cn.items():
        for key, ref in st.items():
            if torch.is_tensor(ref):
                assert torch.equal(c2[i][key], ref), f"state {i} {key} differs between fused and NCCL"
            else:
                assert c2[i][key] == ref
