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
