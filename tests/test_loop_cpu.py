"""training_loop behaviour on CPU: MLP workload, resume equivalence, eval cadence, hooks, OOM skip, evacuation."""

import os

import pytest
import torch
import torch.nn as nn

from koochak_b200 import oom as oom_lib
from koochak_b200.core import hooks as hooks_lib
from koochak_b200.loop import training_loop
from koochak_b200.optim import build_optimizer
from koochak_b200.storage import checkpoint as ck
from koochak_b200.utils.nn_utils import apply_wd


def mlp():
    torch.manual_seed(0)
    m = nn.Sequential(nn.Flatten(), nn.Linear(784, 256), nn.ReLU(), nn.Linear(256, 10))
    apply_wd(m)
    return m


class Data:
    """Deterministic batches indexed by position, so a resumed run sees the same stream."""

    def __init__(self, start=0):
        self.start = start

    def __iter__(self):
        i = self.start
        while True:
            g = torch.Generator().manual_seed(1000 + i)
            yield {"x": torch.rand(64, 1, 28, 28, generator=g), "y": torch.randint(0, 10, (64,), generator=g)}
            i += 1


def step_fn(model, batch, ctx):
    return {"loss": nn.functional.cross_entropy(model(batch["x"]), batch["y"]), "acc": torch.tensor(0.5)}


def cfg(out_dir, **kw):
    base = {"max_steps": 12, "log_every": 4, "ckpt_every": 6, "out_dir": str(out_dir), "grad_clip_norm": 1.0,
            "eval_every": 0, "ema": {"decay": 0.999, "offload_to_cpu": False}}
    base.update(kw)
    return base


def test_mlp_adamw_trains_and_checkpoints(tmp_path):
    m = mlp()
    opt = build_optimizer(m, {"name": "adamw", "lr": 1e-3})
    logs = []
    final = training_loop(model=m, dataset=Data(), step_fn=step_fn, optimizer=opt, train_cfg=cfg(tmp_path),
                          hooks={"on_log": [lambda log, ctx: logs.append(log)]})
    assert [l["step"] for l in logs] == [0, 4, 8]
    assert {"loss", "lr", "step_time_s", "grad_norm", "grad_clip_coefficient", "acc"} <= set(logs[0])
    assert final["step"] == 12 and final["next_step"] == 12
    assert sorted(f for f in os.listdir(tmp_path) if f.endswith(".pt") and f.startswith("step")) == \
        ["step000000006.pt", "step000000012.pt"]
    assert "ema" in final and set(final["ema"]["shadow"]) == {n for n, _ in m.named_parameters()}


def test_resume_matches_uninterrupted_run(tmp_path):
    a = mlp()
    oa = build_optimizer(a, {"name": "muon", "lr": 1e-3})
    full = training_loop(model=a, dataset=Data(), step_fn=step_fn, optimizer=oa, train_cfg=cfg(tmp_path / "a"))
    b = mlp()
    ob = build_optimizer(b, {"name": "muon", "lr": 1e-3})
    training_loop(model=b, dataset=Data(), step_fn=step_fn, optimizer=ob, train_cfg=cfg(tmp_path / "b", max_steps=6))
    c = mlp()
    oc = build_optimizer(c, {"name": "muon", "lr": 1e-3})
    sel = ck.resolve_auto_resume(tmp_path / "b")
    assert sel is not None and sel[1]["next_step"] == 6
    resumed = training_loop(model=c, dataset=Data(start=6), step_fn=step_fn, optimizer=oc,
                            train_cfg=cfg(tmp_path / "b"), resume="auto")
    for k, v in full["model"].items():
        assert torch.allclose(v, resumed["model"][k], atol=1e-6), k
    for k, v in full["ema"]["shadow"].items():
        assert torch.allclose(v, resumed["ema"]["shadow"][k], atol=1e-6), k


def test_eval_cadence_and_hook_order(tmp_path):
    m = mlp()
    opt = build_optimizer(m, {"name": "sgd", "lr": 1e-2})
    events = []
    evals = []

    def eval_fn(model, ds, ctx):
        evals.append(ctx["step"])
        return {"val_loss": 1.0}

    hooks = {}
    for ev in ("on_train_start", "on_update_end", "on_step_end", "on_checkpoint", "on_eval_end", "on_train_end"):
        hooks_lib.add(hooks, ev, (lambda name: (lambda *a, **k: events.append(name)))(ev))
    training_loop(model=m, dataset=Data(), step_fn=step_fn, optimizer=opt, eval_dataset=[0], eval_fn=eval_fn,
                  train_cfg=cfg(tmp_path, max_steps=5, eval_every=2, ckpt_every=100), hooks=hooks)
    assert evals == [0, 2, 4]
    assert events[0] == "on_train_start" and events[-1] == "on_train_end"
    assert events.index("on_update_end") < events.index("on_step_end")


def test_step_fn_contract(tmp_path):
    m = mlp()
    opt = build_optimizer(m, {"name": "sgd", "lr": 1e-2})
    with pytest.raises(RuntimeError, match="loss"):
        training_loop(model=m, dataset=Data(), step_fn=lambda *a: {"x": 1}, optimizer=opt, train_cfg=cfg(tmp_path))


def test_oom_skip_in_place_records_and_replays(tmp_path):
    m = mlp()
    opt = build_optimizer(m, {"name": "adamw", "lr": 1e-3})
    calls = {"n": 0}

    def flaky(model, batch, ctx):
        calls["n"] += 1
        if ctx["step"] == 3:
            raise torch.cuda.OutOfMemoryError("CUDA out of memory (simulated)")
        return step_fn(model, batch, ctx)

    ooms = []
    final = training_loop(model=m, dataset=Data(), step_fn=flaky, optimizer=opt,
                          train_cfg=cfg(tmp_path, max_steps=6, oom_recovery={"enabled": True}),
                          hooks={"on_oom": [lambda rec, ctx: ooms.append(rec)]})
    assert ooms and ooms[0]["action"] == oom_lib.SKIP and ooms[0]["phase"] == "step_fn"
    assert final["oom_skipped_steps"] == [3]
    assert oom_lib.recorded_steps(ck.checkpoint_store(tmp_path)) == frozenset({3})


def test_evacuation_request_file_checkpoints_and_exits(tmp_path, monkeypatch):
    ctrl = tmp_path / "ctrl"
    ctrl.mkdir()
    monkeypatch.setenv("KOOCHAK_EVACUATION_DIR", str(ctrl))
    m = mlp()
    opt = build_optimizer(m, {"name": "adamw", "lr": 1e-3})

    def request_at_2(log, ctx):
        if ctx["step"] == 2:
            (ctrl / "requested").touch()

    with pytest.raises(SystemExit) as exc:
        training_loop(model=m, dataset=Data(), step_fn=step_fn, optimizer=opt,
                      train_cfg=cfg(tmp_path / "run", max_steps=50, evacuation_enabled=True),
                      hooks={"on_update_end": [request_at_2]})
    assert exc.value.code == 75
    assert (ctrl / "evacuated").exists()
    sel = ck.resolve_auto_resume(tmp_path / "run")
    assert sel[1]["step"] == 3 and sel[1]["next_step"] == 3
