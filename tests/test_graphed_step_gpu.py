"""Training through a captured CUDA graph (``train.cuda_graph_step``) matches the eager loop.

GPT-2 (small shape) for 8 updates with Muon + AdamW, EMA and clipping, once
eagerly and once with forward and backward captured after 3 eager updates:
the losses and final parameters agree to a loose tolerance (weight gradients
are summed with fp32 atomics, so two runs are not bitwise equal, and AdamW
with a tiny eps turns such differences in near-zero gradients into steps of
+-lr on a few elements, and Muon's orthogonalisation lifts noise in weak
gradient directions; the key bias, whose exact gradient is zero, is left
out), the graph was captured once and replayed, and the
library's launch counter keeps counting the replayed kernels.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _train(tmp_path, graph: bool):
    from koochak_b200.loop import training_loop
    from koochak_b200.models import GPT2
    from koochak_b200.ops import native
    from koochak_b200.optim import build_optimizer

    torch.manual_seed(0)
    model = GPT2(n_layer=2, n_head=4, n_embd=256, vocab_size=1024, block_size=128).cuda()
    opt = build_optimizer(model, {"name": "muon", "lr": 6e-4, "muon_lr": 0.02, "adam_lr": 6e-4})
    g = torch.Generator().manual_seed(1)
    data = [torch.randint(0, 1024, (4, 129), generator=g) for _ in range(8)]
    batches = [{"idx": d[:, :-1].contiguous(), "targets": d[:, 1:].contiguous()} for d in data]
    losses, launches = [], []

    def hook(log, ctx):
        losses.append(float(log["loss"]))
        launches.append(native().launch_count())

    cfg = {"max_steps": 8, "log_every": 10 ** 6, "eval_every": 0, "ckpt_every": 10 ** 6, "amp": "bf16",
           "grad_clip_norm": 1.0, "out_dir": str(tmp_path / ("g" if graph else "e")), "keep_last_k": 1,
           "ema": {"enabled": True, "decay": 0.99, "offload_to_cpu": False}, "cuda_graph_step": graph,
           "cuda_graph_warmup": 3}
    training_loop(model=model, dataset=iter(batches), step_fn=lambda m, b, c: {"loss": m(b["idx"], b["targets"])},
                  optimizer=opt, train_cfg=cfg, hooks={"on_update_end": [hook]})
    return model, losses, launches


def _comparable(name: str, t: torch.Tensor) -> torch.Tensor:
    if name.endswith("attn.c_attn.bias"):  # the key third's exact gradient is zero (see above)
        C = t.numel() // 3
        return torch.cat([t[:C], t[2 * C:]])
    return t


def test_replayed_gradients_match_eager_gradients():
    """Each replay's loss and gradients equal an eager forward/backward of the same batch and weights.

    The weights are changed in place between replays (as an optimizer step
    does), so the replay must also see refreshed 16-bit weight copies.
    """

    from koochak_b200.models import GPT2
    from koochak_b200.runtime.graphed_step import GraphedStep

    torch.manual_seed(0)
    model = GPT2(n_layer=2, n_head=4, n_embd=256, vocab_size=1024, block_size=128).cuda()
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    gen = torch.Generator().manual_seed(2)

    def batch():
        d = torch.randint(0, 1024, (4, 129), generator=gen).cuda()
        return {"idx": d[:, :-1].contiguous(), "targets": d[:, 1:].contiguous()}

    step = GraphedStep(model, warmup=1)

    def forward(b):
        loss = model(b["idx"], b["targets"])
        return {"loss": loss}, loss, loss

    def eager(b):
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16), step.on_side_stream():
            _, loss, scaled = forward(b)
            scaled.backward()
        return float(loss), {n: p.grad.detach().clone() for n, p in named}

    def rel(a, b):
        return float((a - b).norm() / (b.norm() + 1e-12))

    eager(batch())
    step.note_eager()
    for i in range(4):  # capture, then three replays
        b = batch()
        ref_loss, ref = eager(b)
        _, ref2 = eager(b)  # the same backward again: its spread is the run-to-run noise (fp32 atomics)
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16), step.on_side_stream():
            _, loss = step.run(b, forward)
        assert abs(float(loss) - ref_loss) <= 2e-3 * max(1.0, abs(ref_loss)), (i, float(loss), ref_loss)
        for n, p in named:
            assert p.grad is not None, n
            got, want = _comparable(n, p.grad.detach()), _comparable(n, ref[n])
            noise = rel(_comparable(n, ref2[n]), want)
            err = rel(got, want)
            assert err < max(2e-2, 4 * noise), (i, n, err, noise)
        with torch.no_grad():  # an optimizer-like in-place change of every weight (small: the model stays well
            for _, p in named:  # conditioned, so rounding noise is not amplified)
                p.mul_(0.99).add_(torch.randn_like(p), alpha=1e-3)
    assert step.graph is not None and not step.disabled


def test_graphed_step_matches_eager(tmp_path, monkeypatch):
    from koochak_b200.runtime.graphed_step import GraphedStep

    m_eager, l_eager, _ = _train(tmp_path, False)
    calls = {"capture": 0, "replay": 0}
    capture, run = GraphedStep._capture, GraphedStep.run

    def counted_capture(self, *a, **k):
        calls["capture"] += 1
        return capture(self, *a, **k)

    def counted_run(self, *a, **k):
        calls["replay"] += 1
        return run(self, *a, **k)

    monkeypatch.setattr(GraphedStep, "_capture", counted_capture)
    monkeypatch.setattr(GraphedStep, "run", counted_run)
    m_graph, l_graph, launches = _train(tmp_path, True)
    assert calls == {"capture": 1, "replay": 5}  # updates 3..7 through the graph
    assert len(l_eager) == len(l_graph) == 8
    for a, b in zip(l_eager, l_graph):
        assert abs(a - b) <= 1e-2 * max(1.0, abs(a)), (l_eager, l_graph)
    for (n, p), q in zip(m_eager.named_parameters(), m_graph.parameters()):
        p, q = p.detach(), q.detach()
        if n.endswith("attn.c_attn.bias"):
            # The key third of the QKV bias gets a gradient that is zero in exact arithmetic (a shift of every
            # key by one vector adds a constant to each softmax row); what it receives is fp32 rounding noise of
            # random sign, which AdamW turns into steps of +-lr. Only the query and value thirds are compared.
            C = p.numel() // 3
            p, q = torch.cat([p[:C], p[2 * C:]]), torch.cat([q[:C], q[2 * C:]])
        # AdamW parameters that start at zero (biases) stay small, so +-lr noise steps weigh heavily there;
        # Newton-Schulz gives every singular direction of a Muon update about the same size, so rounding noise
        # in the weak directions of a gradient becomes a visible part of the update. The gradients themselves
        # are compared tightly in test_replayed_gradients_match_eager_gradients.
        err = float((p - q).norm() / (p.norm() + 1e-6))
        assert err < 0.1, (n, err)
    per_update = [b - a for a, b in zip(launches, launches[1:])]
    # every replayed update still counts its kernels (forward/backward from the graph + the eager rest)
    assert all(n > 0 for n in per_update) and max(per_update[4:]) >= 0.5 * max(per_update[:2])

