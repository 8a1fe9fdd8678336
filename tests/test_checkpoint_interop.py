"""Checkpoints move between this runtime and the reference, in both directions.

The reference is the unmodified package installed under ``baseline/_ref``
(skipped when it is not installed). One run directory is shared:

1. this runtime trains the MNIST-shaped MLP for 4 updates (AdamW, EMA, clip,
   checkpoint every 2) and publishes ``step000000004.pt`` + manifest;
2. the reference's own ``resolve_auto_resume`` accepts that checkpoint, and
   the reference's ``training_loop(resume="auto")`` continues from it to
   update 6 and publishes its own checkpoint;
3. this runtime's ``resolve_auto_resume`` accepts the reference's checkpoint
   and its ``training_loop(resume="auto")`` continues to update 8.

Each side checks the cursor it resumed at and that the model weights it
loaded are the ones the other side saved.
"""

from __future__ import annotations

import multiprocessing as mp
import os

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
SHIMS = os.path.join(ROOT, "baseline", "shims")

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "koochak")),
                                reason="reference not installed under baseline/_ref")


def _cfg(steps, out_dir):
    return {"max_steps": steps, "log_every": 1000, "eval_every": 0, "ckpt_every": 2, "grad_clip_norm": 1.0,
            "amp": "fp32", "out_dir": out_dir, "keep_last_k": 5, "device": "cpu",
            "ema": {"enabled": True, "decay": 0.99, "offload_to_cpu": False}}


def _reference_side(out_dir, result):
    import sys

    sys.path[:0] = [REF, SHIMS, ROOT]
    try:
        from examples.mnist.main import SyntheticMNIST, build_model, step_fn
        from koochak.loop import training_loop
        from koochak.storage.checkpoint import resolve_auto_resume

        found = resolve_auto_resume(out_dir)
        if found is None:
            result.put(("FAIL", "reference rejected this runtime's checkpoint"))
            return
        path, ckpt = found
        torch.manual_seed(0)
        model = build_model()
        opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
        seen = []
        training_loop(model=model, dataset=SyntheticMNIST(64, seed=3), step_fn=step_fn, optimizer=opt,
                      train_cfg=_cfg(6, out_dir), resume="auto",
                      hooks={"on_step_end": [lambda logs, ctx: seen.append(int(ctx["step"]))]})
        result.put(("ok", os.path.basename(path), ckpt["next_step"], seen))
    except Exception as exc:  # reported to the parent
        import traceback

        result.put(("FAIL", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()}"))


def _ours(steps, out_dir, resume):
    from examples.mnist.main import SyntheticMNIST, build_model, step_fn
    from koochak_b200.loop import training_loop

    torch.manual_seed(0)
    model = build_model()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    seen = []
    training_loop(model=model, dataset=SyntheticMNIST(64, seed=3), step_fn=step_fn, optimizer=opt,
                  train_cfg=_cfg(steps, out_dir), resume=resume,
                  hooks={"on_step_end": [lambda logs, ctx: seen.append(int(ctx["step"]))]})
    return model, seen


def test_checkpoints_resume_across_frameworks(tmp_path):
    out = str(tmp_path / "run")
    from koochak_b200.storage import checkpoint as ours_ck

    model, seen = _ours(4, out, "none")
    assert seen == [0, 1, 2, 3]
    mine = torch.load(os.path.join(out, "step000000004.pt"), weights_only=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_reference_side, args=(out, q))
    p.start()
    p.join(timeout=300)
    status = q.get(timeout=10)
    assert status[0] == "ok", status[1]
    _, name, next_step, ref_seen = status
    assert name == "step000000004.pt" and next_step == 4 and ref_seen == [4, 5]
    # The reference's checkpoint carries on from the weights this runtime saved.
    theirs = torch.load(os.path.join(out, "step000000006.pt"), weights_only=False)
    assert theirs["next_step"] == 6 and set(theirs) >= {"model", "optimizer", "rng", "ema", "next_step", "step"}
    assert not torch.equal(theirs["model"]["fc1.weight"], mine["model"]["fc1.weight"])
    found = ours_ck.resolve_auto_resume(out)
    assert found is not None and os.path.basename(found[0]) == "step000000006.pt"
    model, seen = _ours(8, out, "auto")
    assert seen == [6, 7]
    final = torch.load(os.path.join(out, "step000000008.pt"), weights_only=False)
    assert final["next_step"] == 8 and final["optimizer"]["state"][0]["step"] == theirs["optimizer"]["state"][0][
        "step"] + 2
