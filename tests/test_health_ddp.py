"""The background GPU-health monitor inside a 2-rank (gloo, CPU) training run.

Rank 0 leads the node and polls both ranks' GPUs through a fake query; a
fault appears after the first poll (a slow SM clock on rank 1's GPU, a query
that raises, or a monitor that stops answering). Expected, as in the
reference (koochak tests/test_background_gpu_health_ddp.py):

* both ranks leave with exit code 42 after the same completed update;
* the monitor thread has stopped;
* the collectives are exactly: one gather at start (leader election), one
  2-element int64 stop-flag reduction per completed update, one gather of the
  failure details once the stop is agreed, one gather of every rank's RNG
  state for the emergency checkpoint -- the monitor adds nothing per step;
* the checkpoint at the agreed cursor holds both ranks' RNG and the failure.
"""

from __future__ import annotations

import json
import multiprocessing as mp
import time
from pathlib import Path

import pytest
import torch


def _worker(rank, init_file, out_dir, results, fault):
    torch.distributed.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=2)
    import koochak_b200.loop as loop_mod
    from koochak_b200.health.background import BackgroundGpuHealth
    from koochak_b200.health.gpu import PRIMARY_QUERY_FIELDS, sample_from_nvidia_smi_row

    made = []

    def fake_query(watchdogs, step, **_):
        assert rank == 0, "only the node leader queries"
        with (Path(out_dir) / f"queries-rank{rank}.jsonl").open("a") as fh:
            fh.write(json.dumps({"step": step, "ranks": [w.rank for w in watchdogs]}) + "\n")
        if fault == "stale":
            made[0]._stop.wait(2)
        elif fault == "query" and step >= 1:
            raise OSError("query failed on purpose")
        rows = []
        for w in watchdogs:
            v = {"index": str(w.rank), "uuid": w.gpu_query_id, "name": "B200", "temperature.gpu": "60",
                 "temperature.memory": "65", "clocks.sm": "1900", "clocks.max.sm": "1965", "utilization.gpu": "100"}
            if fault == "hardware" and w.rank == 1 and step >= 1:
                v["clocks.sm"] = "100"
            rows.append(sample_from_nvidia_smi_row(step=step, rank=w.rank, world_size=2, hostname=w.hostname,
                                                   slurm_node=w.slurm_node, cuda_device=w.cuda_device,
                                                   gpu_query_id=w.gpu_query_id, fields=PRIMARY_QUERY_FIELDS,
                                                   row=[v.get(f, "N/A") for f in PRIMARY_QUERY_FIELDS]))
        return rows

    class TestMonitor(BackgroundGpuHealth):
        interval_seconds = 0.02
        max_sample_age_seconds = 0.5
        query_node = staticmethod(fake_query)
        read_uuid = staticmethod(lambda device: f"GPU-00000000-0000-0000-0000-{rank:012d}")

        def __init__(self, **kw):
            super().__init__(**kw)
            self.enabled = True
            self.device = torch.device("cuda", rank)
            self.cuda_device = rank
            made.append(self)

    loop_mod.BackgroundGpuHealth = TestMonitor
    Path(out_dir).mkdir(exist_ok=True)
    seen = []
    real_reduce, real_gather = torch.distributed.all_reduce, torch.distributed.all_gather_object

    def reduce(t, *a, **k):
        seen.append(("reduce", t.numel(), str(t.dtype)))
        return real_reduce(t, *a, **k)

    def gather(*a, **k):
        seen.append(("gather",))
        return real_gather(*a, **k)

    torch.distributed.all_reduce = reduce
    torch.distributed.all_gather_object = gather
    done = []
    try:
        torch.manual_seed(100 + rank)
        model = torch.nn.Linear(1, 1)
        opt = torch.optim.SGD(model.parameters(), lr=0.1)

        def step_fn(module, batch, ctx):
            time.sleep(0.02)
            return {"loss": module(batch).square().sum()}

        try:
            loop_mod.training_loop(model=model, optimizer=opt, dataset=[torch.ones(1, 1)] * 30, step_fn=step_fn,
                                   train_cfg={"device": "cpu", "ddp": True, "warn_unsharded": False, "max_steps": 30,
                                              "ckpt_every": 100, "log_every": 100, "out_dir": out_dir},
                                   hooks={"on_step_end": [lambda logs, ctx: done.append(ctx["step"])]})
        except SystemExit as exc:
            stop_flags = [s for s in seen if s[0] == "gather" or s[2] == "torch.int64"]
            results.put({"rank": rank, "exit": exc.code, "completed": done, "collectives": stop_flags,
                         "thread_alive": bool(made[0]._thread and made[0]._thread.is_alive())})
        else:
            results.put({"rank": rank, "exit": None})
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("fault", ["hardware", "query", "stale"])
def test_monitor_fault_stops_every_rank_at_one_update(tmp_path, fault):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    out_dir = tmp_path / "run"
    procs = [ctx.Process(target=_worker, args=(r, str(tmp_path / "init"), str(out_dir), results, fault))
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=60)
        assert all(p.exitcode == 0 for p in procs)
        got = sorted((results.get(timeout=5) for _ in procs), key=lambda r: r["rank"])
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
    assert [g["exit"] for g in got] == [42, 42]
    assert got[0]["completed"] == got[1]["completed"]
    assert not any(g["thread_alive"] for g in got)
    for g in got:
        assert g["collectives"] == ([("gather",)] + [("reduce", 2, "torch.int64")] * len(g["completed"])
                                    + [("gather",), ("gather",)])
    from koochak_b200.storage import checkpoint

    cursor = got[0]["completed"][-1] + 1
    saved = checkpoint.load(str(out_dir / f"step{cursor:09d}.pt"))
    assert saved["step"] == saved["next_step"] == cursor and len(saved["rng"]["per_rank"]) == 2
    reason = {"hardware": "sm_clock_low", "query": "monitor_query_failed", "stale": "monitor_stale"}[fault]
    assert saved["metrics"]["gpu_health"]["failures"][0]["reasons"] == [reason]
    assert not (out_dir / "queries-rank1.jsonl").exists()
    rows = [json.loads(x) for x in (out_dir / "queries-rank0.jsonl").read_text().splitlines()]
    assert rows and all(r["ranks"] == [0, 1] for r in rows)
