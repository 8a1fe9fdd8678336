"""Optimizer kernels at the benchmark models' shapes, against PyTorch formulas.

* Batched Newton-Schulz (5 quintic iterations on tcgen05) on GPT-2 124M
  (24 x 768 x 3072) and Llama-style 1.3B (3 x 2048 x 5504) batches, against
  the same iteration in fp32 PyTorch: the relative error must be within
  bf16 precision -- no larger than what PyTorch's own bf16 iteration (the
  reference's arithmetic) shows against fp32, plus a small margin.
* NorMuon (row second moments and per-row scales in native kernels, both the
  plain and the transposed orientation) against the reference formula
  (``normuon_update``) run with PyTorch ops, over two steps.
* Hyperball projection (native, two launches for all matrices) against the
  PyTorch projection, sphere and ball.
"""

from __future__ import annotations

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ns_fp32(X: torch.Tensor, steps: int = 5) -> torch.Tensor:
    from koochak_b200.optim.muon import NS_COEFFS

    a, b, c = NS_COEFFS
    X = X.float()
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * A @ A
        X = a * X + B @ X
    return X


def _ns_torch_bf16(X: torch.Tensor, steps: int = 5) -> torch.Tensor:
    from koochak_b200.optim.muon import NS_COEFFS

    a, b, c = NS_COEFFS
    X = X.bfloat16()
    for _ in range(steps):
        A = X @ X.mT
        B = b * A + c * A @ A
        X = a * X + B @ X
    return X


@pytest.mark.parametrize("n,r,c", [(24, 768, 3072), (3, 2048, 5504), (12, 768, 768)])
def test_newton_schulz_batched_model_shapes(n, r, c):
    from koochak_b200.optim.muon import newton_schulz_batched

    torch.manual_seed(0)
    G = torch.randn(n, r, c, device="cuda")
    X0 = (G / (G.norm(dim=(-2, -1), keepdim=True) + 1e-7)).bfloat16()
    ref = _ns_fp32(X0)
    ours = newton_schulz_batched(X0.clone(), 5).float()
    theirs = _ns_torch_bf16(X0).float()

    def rel(a):
        return float(((a - ref).norm(dim=(-2, -1)) / ref.norm(dim=(-2, -1))).max())

    assert rel(ours) <= 1.25 * rel(theirs) + 2e-3, f"native {rel(ours):.4f} vs torch bf16 {rel(theirs):.4f}"


def _normuon_fp32(grad, momentum, second, beta=0.95, beta2=0.95):
    """NorMuon's update (reference koochak/optim/muon.py:50-74) with the Newton-Schulz iteration in fp32."""

    momentum.lerp_(grad, 1 - beta)
    update = grad.lerp_(momentum, beta)
    rows, cols = update.shape
    X = update.float()
    if rows > cols:
        X = X.mT
    X = X / (X.norm() + 1e-7)
    X = _ns_fp32(X)
    if rows > cols:
        X = X.mT
    vnorm = X.norm()
    second.lerp_((X * X).mean(dim=-1, keepdim=True), 1 - beta2)
    X = X / (second.sqrt() + 1e-10)
    X = X * (vnorm / (X.norm() + 1e-10))
    return X * max(1, rows / cols) ** 0.5


@pytest.mark.parametrize("shape", [(256, 768), (768, 256), (512, 1376)])
def test_normuon_native_matches_reference_formula(shape):
    """Native NorMuon against the formula with an fp32 Newton-Schulz (the oracle), over two steps.

    The Newton-Schulz iteration in bf16 is only accurate to a few percent per
    element, so the native result (tcgen05 bf16 iteration) must be as close to
    the oracle as the reference's own bf16 arithmetic (``normuon_update`` run
    with PyTorch ops) is, with a margin -- for the parameters and for the
    row second moments.
    """

    from koochak_b200.optim.muon import SingleDeviceNorMuonWithAuxAdam, normuon_update

    torch.manual_seed(1)
    mats = [torch.randn(shape, device="cuda") * 0.02 for _ in range(3)]
    native_p = [torch.nn.Parameter(m.clone()) for m in mats]
    opt = SingleDeviceNorMuonWithAuxAdam([dict(params=native_p, use_muon=True, lr=0.02, weight_decay=0.01)])
    arms = {}
    for arm in ("oracle", "torch_bf16"):
        arms[arm] = dict(p=[m.clone() for m in mats], mom=[torch.zeros_like(m) for m in mats],
                         second=[torch.zeros((shape[0], 1), device="cuda") for _ in mats])
    for step in range(2):
        g = torch.Generator(device="cpu").manual_seed(10 + step)
        grads = [torch.randn(shape, generator=g).cuda() for _ in mats]
        for p, gr in zip(native_p, grads):
            p.grad = gr.clone()
        opt.step()
        for arm, st in arms.items():
            fn = _normuon_fp32 if arm == "oracle" else normuon_update
            for i, gr in enumerate(grads):
                upd = fn(gr.clone(), st["mom"][i], st["second"][i], beta=0.95, beta2=0.95)
                st["p"][i].mul_(1 - 0.02 * 0.01)
                st["p"][i].add_(upd.reshape(shape), alpha=-0.02)

    def rel(a, b):
        return float((a - b).norm() / b.norm())

    oracle, theirs = arms["oracle"], arms["torch_bf16"]
    for i in range(len(mats)):
        moved = oracle["p"][i] - mats[i]
        ours_err = rel(native_p[i].detach() - mats[i], moved)
        ref_err = rel(theirs["p"][i] - mats[i], moved)
        assert ours_err <= 1.5 * ref_err + 0.01, f"matrix {i}: update error {ours_err:.4f} vs bf16 torch {ref_err:.4f}"
        sec = opt.state[native_p[i]]["second_momentum_buffer"]
        ours_err = rel(sec, oracle["second"][i])
        ref_err = rel(theirs["second"][i], oracle["second"][i])
        assert ours_err <= 1.5 * ref_err + 0.01, f"matrix {i}: second moment {ours_err:.4f} vs bf16 torch {ref_err:.4f}"


@pytest.mark.parametrize("projection", ["sphere", "ball"])
def test_hyperball_native_matches_torch(projection):
    from koochak_b200.optim.muon import HyperballOptimizer

    torch.manual_seed(2)
    ps = [torch.nn.Parameter(torch.randn(s, device="cuda")) for s in [(768, 768), (256, 3072), (64, 64)]]
    inner = torch.optim.SGD(ps, lr=0.5)
    opt = HyperballOptimizer(inner, ps, projection=projection, radius_scale=0.8)
    twin = [torch.nn.Parameter(p.detach().clone().cpu()) for p in ps]
    twin_opt = HyperballOptimizer(torch.optim.SGD(twin, lr=0.5), twin, projection=projection, radius_scale=0.8)
    for p, q in zip(ps, twin):
        p.grad = torch.randn_like(p)
        q.grad = p.grad.detach().cpu()
    opt.step()
    twin_opt.step()
    for p, q in zip(ps, twin):
        torch.testing.assert_close(p.detach().cpu(), q.detach(), rtol=2e-6, atol=1e-7)


def test_fused_adamw_matches_torch_adamw():
    """build_optimizer('adamw') on CUDA is the native multi-tensor AdamW; three steps against torch.optim.AdamW."""

    from koochak_b200.optim import FusedAdamW, build_optimizer

    torch.manual_seed(3)
    shapes = [(768, 768), (3072,), (1, 197, 768), (1000, 768)]
    ours = [torch.nn.Parameter(torch.randn(s, device="cuda") * 0.02) for s in shapes]
    theirs = [torch.nn.Parameter(p.detach().clone()) for p in ours]
    opt = build_optimizer(ours, {"name": "adamw", "lr": 1e-3, "weight_decay": 0.05})
    assert isinstance(opt, FusedAdamW)
    ref = torch.optim.AdamW(theirs, lr=1e-3, weight_decay=0.05)
    for step in range(3):
        for p, q in zip(ours, theirs):
            g = torch.randn_like(p) * (10.0 ** -step)
            p.grad = g.clone()
            q.grad = g.clone()
        opt.step()
        ref.step()
    for p, q in zip(ours, theirs):
        torch.testing.assert_close(p.detach(), q.detach(), rtol=1e-5, atol=1e-7)
        torch.testing.assert_close(opt.state[p]["exp_avg_sq"], ref.state[q]["exp_avg_sq"], rtol=1e-4, atol=1e-12)
    # The state dict loads into torch.optim.AdamW (same keys per parameter).
    twin = torch.optim.AdamW(theirs, lr=1e-3, weight_decay=0.05)
    twin.load_state_dict(opt.state_dict())
    assert int(twin.state[theirs[0]]["step"]) == 3


def _snapshot(opt, params):
    st = {id(p): {k: (v.clone() if torch.is_tensor(v) else v) for k, v in opt.state[p].items()} for p in params
          if p in opt.state}
    return [p.detach().clone() for p in params], st


@pytest.mark.parametrize("kind", ["adamw", "muon", "normuon"])
def test_device_skip_leaves_state_untouched(kind):
    """A step whose device skip flag is set changes no parameter or optimizer state; the host counters roll back."""

    from koochak_b200.optim import FusedAdamW
    from koochak_b200.optim.muon import SingleDeviceMuonWithAuxAdam, SingleDeviceNorMuonWithAuxAdam

    torch.manual_seed(4)
    mats = [torch.nn.Parameter(torch.randn(s, device="cuda") * 0.02) for s in [(256, 768), (768, 256)]]
    vecs = [torch.nn.Parameter(torch.randn(s, device="cuda") * 0.02) for s in [(768,), (1000, 64)]]
    if kind == "adamw":
        opt = FusedAdamW(mats + vecs, lr=1e-3, weight_decay=0.05)
    else:
        cls = SingleDeviceMuonWithAuxAdam if kind == "muon" else SingleDeviceNorMuonWithAuxAdam
        opt = cls([dict(params=mats, use_muon=True, lr=0.02, weight_decay=0.01),
                   dict(params=vecs, use_muon=False, lr=1e-3, weight_decay=0.0)])
    params = mats + vecs
    for p in params:
        p.grad = torch.randn_like(p)
    opt.step()  # state exists from here on
    before, st_before = _snapshot(opt, params)
    for p in params:
        p.grad = torch.randn_like(p)
    opt.kb_skip = torch.ones(1, device="cuda")
    opt.step()
    torch.cuda.synchronize()
    for p, b in zip(params, before):
        assert torch.equal(p.detach(), b)
    for p in params:
        for k, v in st_before.get(id(p), {}).items():
            if torch.is_tensor(v):
                assert torch.equal(opt.state[p][k], v), k
    opt.kb_rollback_step()
    for p in params:
        if "step" in st_before.get(id(p), {}):
            assert int(opt.state[p]["step"]) == int(st_before[id(p)]["step"])
    # GradScaler's hand-over (found_inf attribute) skips the same way
    opt.found_inf = torch.ones((), device="cuda")
    opt.step()
    del opt.found_inf
    torch.cuda.synchronize()
    for p, b in zip(params, before):
        assert torch.equal(p.detach(), b)


def test_deferred_gate_matches_synchronous_gate_and_raises_like_the_reference():
    """The two-phase gate (optimizer enqueued before the statistics are read) gives the synchronous gate's
    parameters bit for bit; with a non-finite gradient under clipping it raises FloatingPointError and leaves
    parameters and Adam step counters as they were."""

    from koochak_b200.core.precision import NoOpScaler
    from koochak_b200.models import GPT2
    from koochak_b200.optim import build_optimizer
    from koochak_b200.runtime.gate import GradientGate

    def make():
        torch.manual_seed(0)
        m = GPT2(n_layer=2, n_head=4, n_embd=256, vocab_size=512, block_size=128).cuda()
        return m, build_optimizer(m, {"name": "muon", "lr": 6e-4, "muon_lr": 0.02})

    idx = torch.randint(0, 512, (4, 128), device="cuda")
    # Same gradients into both runs (the backward's fp32 weight-gradient reductions are not bitwise
    # reproducible between two backward passes): model a computes them, model b gets a copy.
    (ma, oa), (mb, ob) = make(), make()
    gates = [GradientGate(max_norm=0.5, check_every=0, scaler=NoOpScaler(), profile=lambda k, f: f())
             for _ in range(2)]
    for _ in range(3):
        oa.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = ma(idx, idx)
        loss.backward()
        for pa, pb in zip(ma.parameters(), mb.parameters()):
            pb.grad = pa.grad.clone()
        for gate, m, opt, defer in ((gates[0], ma, oa, True), (gates[1], mb, ob, False)):
            gate.begin(m, opt, 0, True, defer=defer)
            opt.step()
            out = gate.finish(m, opt)
            assert 0.0 < out["grad_norm"] and 0.0 < out["grad_clip_coefficient"] <= 1.0
    for a, b in zip(ma.parameters(), mb.parameters()):
        assert torch.equal(a.detach(), b.detach())

    m, opt = make()
    gate = GradientGate(max_norm=0.5, check_every=0, scaler=NoOpScaler(), profile=lambda k, f: f())
    with torch.autocast("cuda", dtype=torch.bfloat16):
        m(idx, idx).backward()
    gate.begin(m, opt, 0, True)
    opt.step()
    gate.finish(m, opt)
    before = [p.detach().clone() for p in m.parameters()]
    steps = {id(p): int(st["step"]) for p, st in opt.state.items() if "step" in st}
    opt.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        m(idx, idx).backward()
    next(iter(m.parameters())).grad[0, 0] = float("inf")
    gate.begin(m, opt, 1, True)
    opt.step()
    with pytest.raises(FloatingPointError):
        gate.finish(m, opt)
    for p, b in zip(m.parameters(), before):
        assert torch.equal(p.detach(), b)
    for p, st in opt.state.items():
        if "step" in st:
            assert int(st["step"]) == steps[id(p)]
