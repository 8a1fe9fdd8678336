"""Logging sinks, W&B key mapping (with a fake wandb module) and coordinator events."""

from __future__ import annotations

import io
import json
import sys
import types
import warnings

import pytest

from koochak_b200.core.hooks import emit, merge
from koochak_b200.logging import (CSVLogger, log_step_tsv, make_csv_hooks, make_jsonl_hooks, make_stdout_hooks)
from koochak_b200.logging.events import (CheckpointArtifactAckRejected, CheckpointArtifactAckTimeout,
                                         checkpoint_event_id, make_event_hooks, make_scruffy_hooks)


def test_tsv_order_and_format():
    buf = io.StringIO()
    log_step_tsv({"zeta": 1.234567, "step": 3, "lr": 0.001, "loss": 2.0, "flag": True, "bad": float("nan")},
                 file=buf)
    assert buf.getvalue().strip().split("\t") == ["step", "3", "loss", "2", "lr", "0.001", "bad", "nan", "flag", "1",
                                                  "zeta", "1.235"]


def test_csv_schema_fixed_by_first_row(tmp_path):
    p = tmp_path / "m.csv"
    lg = CSVLogger(str(p))
    lg.write({"step": 0, "loss": 1.0})
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        lg.write({"step": 1, "loss": 0.5, "extra": 3})
        lg.write({"step": 2, "loss": 0.25, "extra": 4})
    assert len(w) == 1 and "extra" in str(w[0].message)
    lg.close()
    rows = p.read_text().strip().splitlines()
    assert rows == ["step,loss", "0,1.0", "1,0.5", "2,0.25"]


def test_hook_sinks_on_rank0(tmp_path):
    csv_p, jl_p = tmp_path / "a.csv", tmp_path / "a.jsonl"
    buf = io.StringIO()
    hooks = merge(merge(make_csv_hooks(str(csv_p)), make_jsonl_hooks(str(jl_p))), make_stdout_hooks(buf))
    emit(hooks, "on_log", {"step": 0, "loss": 1.5}, {"step": 0})
    emit(hooks, "on_eval_end", {"val_loss": 1.0}, {"step": 0})
    emit(hooks, "on_train_end", {})
    lines = [json.loads(x) for x in jl_p.read_text().splitlines()]
    assert lines == [{"loss": 1.5, "step": 0}, {"step": 0, "val_loss": 1.0}]
    assert "loss\t1.5" in buf.getvalue()
    assert csv_p.read_text().splitlines()[0] == "step,loss"


def _fake_wandb(monkeypatch):
    calls = []
    run = types.SimpleNamespace(summary={}, id="abc", name="run")
    mod = types.ModuleType("wandb")
    mod.Settings = lambda: None
    mod.init = lambda **kw: calls.append(("init", kw))
    mod.log = lambda payload, step=None, commit=True: calls.append(("log", payload, step, commit))
    mod.run = run
    mod.finish = lambda: calls.append(("finish",))
    monkeypatch.setitem(sys.modules, "wandb", mod)
    return calls, run


def test_wandb_hooks_namespacing_and_commit(monkeypatch):
    calls, run = _fake_wandb(monkeypatch)
    from koochak_b200.logging.wandb_logger import make_wandb_hooks, run_id_from_name

    hooks = make_wandb_hooks({"name": "My Run!", "watch_model": False})
    cfg = {"eval_every": 10}
    emit(hooks, "on_train_start", {"train_cfg": cfg}, suppress_exceptions=False)
    assert calls[0][1]["id"] == run_id_from_name("My Run!")
    emit(hooks, "on_log", {"loss": 1.0, "step_time_s": 0.1}, {"step": 10, "train_cfg": cfg}, suppress_exceptions=False)
    assert calls[-1] == ("log", {"train/loss": 1.0, "stats/step_time_s": 0.1}, 10, False)
    emit(hooks, "on_log", {"loss": 1.0}, {"step": 11, "train_cfg": cfg}, suppress_exceptions=False)
    assert calls[-1][3] is True
    emit(hooks, "on_eval_end", {"val_loss": 0.5}, {"step": 10}, suppress_exceptions=False)
    assert calls[-1] == ("log", {"val/loss": 0.5}, 10, True)
    assert run.summary["best/val_loss"] == 0.5


def test_event_hooks_rate_limit_and_failures():
    sent = []
    now = [0.0]
    hooks = make_event_hooks(lambda k, d: sent.append((k, d)), progress_interval_s=30, clock=lambda: now[0])
    ctx = {"train_cfg": {"max_steps": 100}, "world_size": 2, "device": "cuda:0"}
    emit(hooks, "on_train_start", ctx)
    for step in range(5):
        now[0] = step * 10.0
        emit(hooks, "on_step_end", {"loss": 1.0, "lr": 0.1, "junk": "x"}, {**ctx, "step": step})
    progress = [d for k, d in sent if k == "workload.progress"]
    assert [d["step"] for d in progress] == [0, 3]
    assert progress[0]["metrics"] == {"loss": 1.0, "lr": 0.1}
    assert progress[1]["completed"] == 4 and progress[1]["total"] == 100
    emit(hooks, "on_train_end", {**ctx, "step": 4, "evacuation_requested": True})
    assert sent[-1] == ("workload.phase", {"phase": "training", "status": "evacuated", "step": 4})

    def broken(kind, data):
        raise OSError("down")

    hooks = make_event_hooks(broken)
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        emit(hooks, "on_train_start", {})
        emit(hooks, "on_train_end", {})
    assert len(w) == 1


def _checkpoint_with_publication(tmp_path):
    import torch

    from koochak_b200.storage import checkpoint as ck

    path = str(tmp_path / "step000000001.pt")
    ck.save({"model": {"w": torch.zeros(2)}, "step": 1}, path)
    return path, ck.publication(path)


def test_scruffy_hooks_ack_paths(tmp_path, monkeypatch):
    path, pub = _checkpoint_with_publication(tmp_path)
    events = []
    mod = types.ModuleType("scruffy")

    def publish_event(root, *, job_id, kind, data, source, **kw):
        events.append((kind, kw))
        if kind == "workload.artifact":
            if mode[0] == "pending":
                return {"state": "pending"}
            return {"state": mode[0], "acknowledged": mode[0] == "accepted"}
        return None

    mode = ["accepted"]
    mod.publish_event = publish_event
    monkeypatch.setitem(sys.modules, "scruffy", mod)
    monkeypatch.setenv("SCRUFFY_ROOT", str(tmp_path))
    monkeypatch.setenv("SCRUFFY_JOB_ID", "job1")
    hooks = make_scruffy_hooks(artifact_ack_timeout_s=1)
    emit(hooks, "on_checkpoint", path, {}, {"step": 1})
    kind, kw = events[-1]
    assert kw["event_id"] == checkpoint_event_id(pub) and kw["wait"] is True
    mode[0] = "rejected"
    with pytest.raises(CheckpointArtifactAckRejected):
        emit(hooks, "on_checkpoint", path, {}, {"step": 1})
    mode[0] = "pending"  # neither accepted nor rejected, and no way to reconcile
    with pytest.raises(CheckpointArtifactAckTimeout) as ei:
        emit(hooks, "on_checkpoint", path, {}, {"step": 1})
    assert ei.value.exit_code == 76
