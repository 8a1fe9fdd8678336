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

from koochak_b200.parallel.ddp import split_buckets
from koochak_b200.parallel.symm import MODE_ALL, MODE_LOCAL, plan_bucket_chunks, plan_chunks, shard_bounds


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


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("shard_rest", [False, True])
def test_bucket_plan_owners_and_shards(world, shard_rest):
    """Owned tensors are reduced whole by their owner only; the rest split evenly, each element once."""

    sizes = [768, 5, 2304 * 768, 3, 1024, 7, 4096]
    layout, off = [], 0
    for tid, n in enumerate(sizes):
        layout.append((off, n, tid))
        off += (n + 3) // 4 * 4
    owner_of = {2: world - 1, 6: 0}
    covered = torch.zeros(off, dtype=torch.int32)
    for r in range(world):
        for start, length, tid, mode in plan_bucket_chunks(layout, world, r, owner_of, shard_rest, max_chunk=1000):
            o, n, _ = layout[tid]
            assert start % 4 == 0 and 0 < length <= 1000 and o <= start and start + length <= o + n
            if tid in owner_of:
                assert r == owner_of[tid] and mode == MODE_LOCAL
            else:
                assert mode == (MODE_LOCAL if shard_rest else MODE_ALL)
                lo, hi = shard_bounds(n, world, r)
                assert o + lo <= start and start + length <= o + hi, "chunk outside this rank's shard"
            covered[start:start + length] += 1
    for o, n, _ in layout:
        assert bool((covered[o:o + n] == 1).all())


def test_split_buckets_cap_list():
    """Bucket i closes at caps[min(i, len - 1)] elements; a large tensor forms a bucket of its own."""

    assert split_buckets([4, 4, 4, 4, 4], [8]) == [[0, 1], [2, 3], [4]]
    assert split_buckets([4, 4, 4, 4, 4], [4, 12]) == [[0], [1, 2, 3], [4]]
    assert split_buckets([100, 1, 1], [8]) == [[0], [1, 2]]


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
        ok = True
        msgs = []
        modes = "mc" if use_mc else "p2p"
        # (owner_of, shard_rest): plain all-reduce; tensor 1 owned by rank 1 and tensor 3 by rank 0 with the
        # rest reduce-scattered.
        for owner_of, shard_rest in (({}, False), ({1: 1, 3: 0}, True)):
            red = FusedGradReducer(segs, tid, torch.device("cuda", rank), blocks=8, timeout_s=20.0,
                                   use_multicast=use_mc, owner_of=owner_of, shard_rest=shard_rest)
            modes = "mc" if red.ws.mc_base else "p2p"
            for step in range(2):
                red.begin_step()
                scale = torch.tensor([4.0 if step else 1.0], device="cuda")
                expect = {}
                for b, layout in enumerate(red.layouts):
                    for off, n, t in layout:
                        g = torch.Generator(device="cpu").manual_seed(1000 * step + 10 * t)
                        allv = torch.randn(world, n, generator=g)
                        red.buffers[b][off:off + n].copy_(allv[rank].cuda())
                        expect[t] = (b, off, allv.mean(0) / scale.item(), allv[rank])
                    # The ranks launch the same bucket with different grids (rank 1: 4x wider on step 1).
                    red.reduce(b, scale, blocks=8 * (1 + 3 * rank * step))
                gate = red.seal_gate(1.0)
                torch.cuda.synchronize()
                stats = red.current_stats().cpu()
                for t, (b, off, ref, local) in expect.items():
                    n = ref.numel()
                    got = red.buffers[b][off:off + n].cpu()
                    if t in owner_of:
                        want = ref if owner_of[t] == rank else local
                    elif shard_rest:
                        lo, hi = shard_bounds(n, world, rank)
                        want = local.clone()
                        want[lo:hi] = ref[lo:hi]
                    else:
                        want = ref
                    if not torch.allclose(got, want, rtol=1e-5, atol=1e-6):
                        ok = False
                        msgs.append(f"{owner_of} step {step} tensor {t}: max err {(got - want).abs().max():.3g}")
                    ss = float((ref.double() ** 2).sum())
                    if abs(float(stats[t]) - ss) > 1e-3 * ss + 1e-4:
                        ok = False
                        msgs.append(f"{owner_of} step {step} tensor {t}: sumsq {float(stats[t])} vs {ss}")
                norm = float(sum(float((e[2].double() ** 2).sum()) for e in expect.values())) ** 0.5
                g = gate.cpu()
                if abs(float(g[0]) - norm) > 1e-3 * norm or float(g[3]) != 0.0 or float(g[2]) != 0.0:
                    ok = False
                    msgs.append(f"{owner_of} step {step}: gate {g.tolist()} vs norm {norm}")
            # A non-finite value on one rank sets found_inf everywhere.
            red.begin_step()
            for b in range(len(red.buffers)):
                red.buffers[b].zero_()
            if rank == 0:
                red.buffers[1][5] = float("inf")
            for b in range(len(red.buffers)):
                red.reduce(b, None)
            g = red.seal_gate(None).cpu()
            if float(g[2]) != 1.0:
                ok = False
                msgs.append(f"{owner_of}: found_inf not set")
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(("ok " if ok else "FAIL ") + modes + "\n" + "\n".join(msgs))
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
