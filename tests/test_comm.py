"""Fused gradient all-reduce: shard planning on CPU, kernels on 1 and 2 GPUs.

The 2-GPU cases spawn one process per GPU and compare the fused kernel (P2P
and, where the switch offers it, multimem) against the mean of the ranks'
inputs computed in fp32 by PyTorch, including the per-tensor sums of squares
and the found-inf flag. The bounded-wait case waits on a flag that nothing
sets, on one GPU, and checks that the kernel returns with the timeout status.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

from koochak_b200.parallel.symm import plan_chunks, shard_bounds


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shards_cover_bucket_once(world):
    sizes = [768, 5, 2304 * 768, 3, 1024, 7]
    segs, off = [], 0
    for tid, n in enumerate(sizes):
        segs.append((off, n, tid))
        off += (n + 3) // 4 * 4
    covered = torch.zeros(off, dtype=torch.int32)
    for r in range(world):
        lo, hi = shard_bounds(off, world, r)
        assert lo % 4 == 0 and (hi % 4 == 0 or hi == off)
        for start, length, tid in plan_chunks(segs, lo, hi, max_chunk=1000):
            assert start % 4 == 0 and 0 < length <= 1000
            s_off, s_n, _ = segs[tid]
            assert s_off <= start and start + length <= s_off + s_n, "chunk crosses a tensor"
            covered[start:start + length] += 1
    for s_off, s_n, _ in segs:
        assert bool((covered[s_off:s_off + s_n] == 1).all())


@pytest.mark.gpu
def test_barrier_timeout_sets_status():
    """A barrier whose second participant never arrives returns with status 5 (peer timeout)."""

    from koochak_b200.ops import _ext

    C = _ext.native()
    _ext.native().read_and_clear_status(0)
    flags = torch.zeros(128 * 8, dtype=torch.int32, device="cuda")
    base = flags.data_ptr()
    # World of two whose "peer" is this same buffer: rank 1's slot is never written.
    C.comm_barrier([base, base], 0, 0, 1, 1, 0.2, 0)
    torch.cuda.synchronize()
    assert C.read_and_clear_status(0) == 5
    # The context is still usable afterwards.
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0


def _worker(rank: int, world: int, port: int, use_mc: bool, result_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from koochak_b200.parallel.symm import FusedGradReducer

        sizes = [[1000, 768 * 4, 3], [2304 * 768 + 1, 6]]
        tid = 0
        segs = []
        for bucket in sizes:
            segs.append([(n, tid + i) for i, n in enumerate(bucket)])
            tid += len(bucket)
        red = FusedGradReducer(segs, tid, torch.device("cuda", rank), blocks=8, timeout_s=20.0,
                               use_multicast=use_mc)
        mode = "mc" if red.ws.mc_base else "p2p"
        ok = True
        msgs = []
        for step in range(2):
            red.begin_step()
            scale = torch.tensor([4.0 if step else 1.0], device="cuda")
            expect = {}
            for b, layout in enumerate(red.layouts):
                for off, n, t in layout:
                    g = torch.Generator(device="cpu").manual_seed(1000 * step + 10 * t)
                    allv = torch.randn(world, n, generator=g)
                    red.buffers[b][off:off + n].copy_(allv[rank].cuda())
                    expect[t] = (b, off, allv.mean(0) / scale.item())
                # Second step: the last bucket runs on a wider grid than the rest (as after backward).
                red.reduce(b, scale, blocks=32 if step == 1 and b == len(red.layouts) - 1 else None)
            torch.cuda.synchronize()
            stats = red.current_stats().cpu()
            for t, (b, off, ref) in expect.items():
                got = red.buffers[b][off:off + ref.numel()].cpu()
                if not torch.allclose(got, ref, rtol=1e-5, atol=1e-6):
                    ok = False
                    msgs.append(f"step {step} tensor {t}: max err {(got - ref).abs().max():.3g}")
                ss = float((ref.double() ** 2).sum())
                if abs(float(stats[t]) - ss) > 1e-3 * ss + 1e-4:
                    ok = False
                    msgs.append(f"step {step} tensor {t}: sumsq {float(stats[t])} vs {ss}")
            if float(stats[tid]) != 0.0:
                ok = False
                msgs.append("found_inf set on finite data")
        gate = red.gate(1.0).cpu()
        if float(gate[3]) != 0.0:
            ok = False
            msgs.append(f"status {float(gate[3])}")
        # A non-finite value on one rank sets found_inf everywhere.
        red.begin_step()
        for b in range(len(red.buffers)):
            red.buffers[b].zero_()
        if rank == 0:
            red.buffers[1][5] = float("inf")
        for b in range(len(red.buffers)):
            red.reduce(b, None)
        torch.cuda.synchronize()
        if float(red.current_stats()[tid]) != 1.0:
            ok = False
            msgs.append("found_inf not set")
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(("ok " if ok else "FAIL ") + mode + "\n" + "\n".join(msgs))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("use_mc", [False, True])
def test_fused_allreduce_two_gpus(tmp_path, use_mc):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), use_mc, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        text = (tmp_path / f"rank{r}.txt").read_text()
        assert text.startswith("ok"), text
