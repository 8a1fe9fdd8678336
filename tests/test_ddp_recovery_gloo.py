"""Evacuation and OOM replay across data-parallel ranks (two gloo processes on CPU).

Behaviours of the reference's DDP tests (tests/test_interruption.py:48-83,
472-556 and tests/test_oom_recovery.py:292-350), run against this runtime:

* an evacuation requested on one rank is agreed on at the next update
  boundary: both ranks exit with code 75 after the same update, and rank 0's
  terminal checkpoint holds every rank's RNG state;
* with an evacuation requested through the runner's directory, the other
  ranks leave only after rank 0 has reported the evacuation (its hook may
  take a while), and the ``evacuated`` marker is written;
* an OOM record written by one rank in an earlier attempt makes every rank
  skip that update on the next attempt, so the ranks stay in step and end
  with identical weights.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import time
from pathlib import Path
from typing import Any

import torch

from koochak_b200.interruption import EVACUATED_FILE, EVACUATION_EXIT_CODE, EVACUATION_REQUEST_FILE


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg(out_dir: str, max_steps: int) -> dict:
    return {"max_steps": max_steps, "log_every": 10 ** 6, "eval_every": 0, "ckpt_every": 10 ** 6,
            "out_dir": out_dir, "keep_last_k": 2, "ddp": True, "warn_unsharded": False, "device": "cpu",
            "evacuation_enabled": True}


def _data(n: int = 8):
    return [{"x": torch.ones(2, 1) * (i + 1), "y": torch.zeros(2, 1)} for i in range(n)]


def _loss(module, batch, ctx):
    return {"loss": torch.nn.functional.mse_loss(module(batch["x"]), batch["y"])}


def _run(rank: int, port: int, fn, *args) -> None:
    torch.distributed.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    try:
        fn(rank, *args)
    finally:
        torch.distributed.destroy_process_group()


def _spawn(fn, *args, timeout: float = 120.0) -> None:
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_run, args=(rank, port, fn, *args)) for rank in range(2)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=timeout)
            assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()


# ----------------------------------------------------------------------------- evacuation on one rank


def _evacuate_on_rank1(rank: int, out_dir: str, q: Any) -> None:
    from koochak_b200.interruption import EvacuationController
    from koochak_b200.loop import training_loop

    torch.manual_seed(7 + rank)
    model = torch.nn.Linear(1, 1, bias=False)
    controller = EvacuationController(False)
    if rank == 1:
        controller.request()
    try:
        training_loop(model=model, dataset=_data(), step_fn=_loss, optimizer=torch.optim.SGD(model.parameters(), lr=0.1),
                      train_cfg=_cfg(out_dir, 4), evacuation=controller)
        q.put((rank, "returned", None))
    except SystemExit as exc:
        q.put((rank, "exit", exc.code))


def test_evacuation_on_one_rank_stops_both_after_the_same_update(tmp_path: Path) -> None:
    from koochak_b200.storage import checkpoint

    q = mp.get_context("spawn").Queue()
    _spawn(_evacuate_on_rank1, str(tmp_path / "run"), q)
    got = sorted(q.get(timeout=10) for _ in range(2))
    assert got == [(0, "exit", EVACUATION_EXIT_CODE), (1, "exit", EVACUATION_EXIT_CODE)]
    saved = checkpoint.load(str(tmp_path / "run" / "step000000001.pt"))
    assert saved["next_step"] == 1
    assert len(saved["rng"]["per_rank"]) == 2


# ----------------------------------------------------------------------------- exit order


def _slow_rank0_report(rank: int, out_dir: str, control: str, q: Any) -> None:
    from koochak_b200.loop import training_loop

    os.environ["KOOCHAK_EVACUATION_DIR"] = control
    model = torch.nn.Linear(1, 1, bias=False)

    def report(*_args: Any) -> None:
        time.sleep(1.0)  # rank 0 waiting for the coordinator's acknowledgement
        q.put((rank, "reported", time.time()))

    try:
        training_loop(model=model, dataset=_data(), step_fn=_loss, optimizer=torch.optim.SGD(model.parameters(), lr=0.1),
                      train_cfg=_cfg(out_dir, 4), hooks={"on_evacuation": [report]})
    except SystemExit as exc:
        q.put((rank, "exit", time.time(), exc.code))


def test_other_ranks_leave_after_rank0_reported_the_evacuation(tmp_path: Path) -> None:
    control = tmp_path / "control"
    control.mkdir()
    (control / EVACUATION_REQUEST_FILE).touch()
    q = mp.get_context("spawn").Queue()
    _spawn(_slow_rank0_report, str(tmp_path / "run"), str(control), q)
    items = [q.get(timeout=10) for _ in range(3)]
    reported = [it[2] for it in items if it[1] == "reported"]
    exits = {it[0]: it for it in items if it[1] == "exit"}
    assert len(reported) == 1
    assert {r: it[3] for r, it in exits.items()} == {0: EVACUATION_EXIT_CODE, 1: EVACUATION_EXIT_CODE}
    assert exits[1][2] >= reported[0]
    assert (control / EVACUATED_FILE).is_file()


# ----------------------------------------------------------------------------- OOM replay


def _replay(rank: int, out_dir: str, q: Any) -> None:
    from koochak_b200.loop import training_loop

    torch.manual_seed(0)
    model = torch.nn.Linear(1, 1, bias=False)
    seen = []

    def step_fn(module, batch, ctx):
        seen.append(int(ctx["step"]))
        x = batch["x"] * (rank + 1)  # different data per rank: weights agree only through the all-reduce
        return {"loss": torch.nn.functional.mse_loss(module(x), batch["y"])}

    final = training_loop(model=model, dataset=iter(_data(64)), step_fn=step_fn,
                          optimizer=torch.optim.SGD(model.parameters(), lr=0.1),
                          train_cfg={**_cfg(out_dir, 4), "oom_recovery": {"enabled": True}})
    q.put((rank, seen, final["model"]["weight"].tolist(), final.get("oom_skipped_steps")))


def test_recorded_oom_step_is_skipped_by_every_rank(tmp_path: Path) -> None:
    from koochak_b200 import oom as oom_lib
    from koochak_b200.storage.store import open_store

    out = tmp_path / "out"
    oom_lib.write_record(open_store(str(out)), {"step": 1, "rank": 1})  # only rank 1 failed there
    q = mp.get_context("spawn").Queue()
    _spawn(_replay, str(out), q)
    got = sorted(q.get(timeout=10) for _ in range(2))
    for _rank, seen, _w, skipped in got:
        assert seen == [0, 2, 3]
        assert skipped == [1]
    assert got[0][2] == got[1][2]
