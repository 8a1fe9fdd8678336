"""Sharded Muon with the parameter all-gather fused into the owner's update kernel.

Each rank runs the distributed ``MuonWithAuxAdam`` on the same parameters and
the same (already averaged) gradients; matrix i of the size-sorted group is
owned by rank i % world (the reference's rule), whose update kernel stores the new matrix into every rank's
copy (P2P stores, or ``multimem.st`` where the switch offers multicast). The
oracle is the single-GPU ``SingleDeviceMuonWithAuxAdam`` on a copy of the
parameters on the same GPU: every rank must end up with the single-GPU result
for every matrix, owned or not, over three steps. The one-GPU case runs the
same path with a single rank that owns every matrix.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SHAPES = [(256, 512)] * 3 + [(512, 256)] * 3 + [(384, 384)] * 2 + [(128, 640), (640, 128)]


def _worker(rank: int, world: int, port: int, use_mc: bool, result_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      KOOCHAK_B200_MULTIMEM="1" if use_mc else "0", KOOCHAK_B200_COMM_TIMEOUT_S="20")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    msgs = []
    mode = "?"
    try:
        from koochak_b200.optim.muon import MuonWithAuxAdam, SingleDeviceMuonWithAuxAdam

        g = torch.Generator(device="cpu").manual_seed(7)
        init = [torch.randn(s, generator=g) * 0.02 for s in SHAPES]
        dist_p = [torch.nn.Parameter(t.clone().to(dev)) for t in init]
        ref_p = [torch.nn.Parameter(t.clone().to(dev)) for t in init]
        for p in dist_p:
            p._kb_shadow = torch.empty(p.shape, device=dev, dtype=torch.bfloat16)
            p._kb_shadow_version = -1
        opt = MuonWithAuxAdam([dict(params=dist_p, use_muon=True, lr=0.02, weight_decay=0.01)])
        if world == 1:
            opt._distributed_now = lambda: True  # one rank owning every matrix: same kernels, local stores only
        ref = SingleDeviceMuonWithAuxAdam([dict(params=ref_p, use_muon=True, lr=0.02, weight_decay=0.01)])
        for step in range(3):
            gs = torch.Generator(device="cpu").manual_seed(100 + step)
            grads = [torch.randn(s, generator=gs) for s in SHAPES]
            for p, q, gr in zip(dist_p, ref_p, grads):
                p.grad = gr.to(dev)
                q.grad = gr.to(dev)
            opt.step()
            ref.step()
            torch.cuda.synchronize()
            for k, (p, q) in enumerate(zip(dist_p, ref_p)):
                err = float((p.detach() - q.detach()).abs().max())
                if not err <= 1e-6:
                    msgs.append(f"step {step} matrix {k} {tuple(p.shape)}: max err {err:.3g}")
        slab = opt.__dict__.get("_kb_slab")
        if slab is None:
            msgs.append("expected a symmetric parameter slab")
        else:
            mode = "mc" if slab.ws.mc_base else "p2p"
            lo = slab.ws.tensor.data_ptr()
            if not all(lo <= p.data_ptr() < lo + slab.ws.nbytes for p in dist_p):
                msgs.append("parameters are not stored in the slab")
        # Ownership follows the reference: index in the size-sorted group mod world.
        order = opt.param_groups[0]["params"]
        for i, p in enumerate(order):
            if ("momentum_buffer" in opt.state[p]) != (i % world == rank):
                msgs.append(f"matrix {i} of the sorted group: momentum on the wrong rank")
        # Owners wrote their bf16 copies; the others are marked for recast.
        for p in dist_p:
            owned = "momentum_buffer" in opt.state[p]
            if owned and not torch.equal(p._kb_shadow, p.detach().bfloat16()):
                msgs.append(f"owner's bf16 copy of {tuple(p.shape)} is stale")
            if world > 1 and not owned and p._kb_shadow_version != -1:
                msgs.append(f"non-owned {tuple(p.shape)} not marked for recast")
        from koochak_b200.ops import native

        status = native().read_and_clear_status(rank)
        if status:
            msgs.append(f"device status {status}")
    except Exception as e:  # reported through the result file
        msgs.append(f"{type(e).__name__}: {e}")
    finally:
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(("FAIL " if msgs else "ok ") + mode + "\n" + "\n".join(msgs))
        dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_muon_gather_one_rank(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(1, _free_port(), False, str(tmp_path)), nprocs=1, join=True)
    text = (tmp_path / "rank0.txt").read_text()
    assert text.startswith("ok"), text


@pytest.mark.gpu
@pytest.mark.parametrize("use_mc", [False, True])
def test_sharded_muon_gather_matches_single_gpu(tmp_path, use_mc):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), use_mc, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        text = (tmp_path / f"rank{r}.txt").read_text()
        assert text.startswith("ok"), text
