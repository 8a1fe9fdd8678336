import math

import pytest
import torch

from koochak_b200.optim import build_optimizer, clip_grad_norm_
from koochak_b200.optim.muon import SingleDeviceMuonWithAuxAdam, muon_update, zeropower_via_newtonschulz5
from koochak_b200.utils.ema import EMA
from koochak_b200.utils.ema_posthoc import gamma_from_srel, ls_coeffs_for_power_profile, srel_from_gamma
from koochak_b200.utils.nn_utils import apply_wd, prepare_param_groups_for_muon, tag_module


def test_clip_matches_torch_and_raises_on_inf():
    torch.manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(5, 3)) for _ in range(3)]
    for p in ps:
        p.grad = torch.randn_like(p) * 10
    ref = [p.grad.clone() for p in ps]
    expected = torch.nn.utils.clip_grad_norm_([torch.nn.Parameter(torch.zeros(1)) for _ in []] or
                                              [type("P", (), {})()] if False else ps, float("inf"))
    stats = clip_grad_norm_(ps, 1.0)
    total = math.sqrt(sum(float((r ** 2).sum()) for r in ref))
    assert abs(stats.norm - total) / total < 1e-6
    assert abs(float(torch.cat([p.grad.flatten() for p in ps]).norm()) - 1.0) < 1e-4
    ps[0].grad[0, 0] = float("nan")
    with pytest.raises(FloatingPointError):
        clip_grad_norm_(ps, 1.0)
    big = [torch.nn.Parameter(torch.zeros(4))]
    big[0].grad = torch.full((4,), 3e38)
    st = clip_grad_norm_(big, 1.0)
    assert st.used_scaled_norm and abs(float(big[0].grad.norm()) - 1.0) < 1e-3


def test_newton_schulz_orthogonalizes():
    torch.manual_seed(1)
    g = torch.randn(64, 96)
    x = zeropower_via_newtonschulz5(g, 5).float()
    s = torch.linalg.svdvals(x)
    assert s.max() < 1.4 and s.min() > 0.4
    tall = zeropower_via_newtonschulz5(torch.randn(96, 64), 5)
    assert tall.shape == (96, 64)


def test_muon_groups_and_state_format():
    model = torch.nn.Sequential(torch.nn.Embedding(10, 8), torch.nn.Linear(8, 16), torch.nn.LayerNorm(16),
                                torch.nn.Linear(16, 4))
    apply_wd(model)
    tag_module(model[0], "mapping")
    groups = prepare_param_groups_for_muon(model, lr=0.1, weight_decay=0.01)
    assert [g["use_muon"] for g in groups] == [False, False, True]
    muon = groups[-1]["params"]
    assert [tuple(p.shape) for p in muon] == sorted([tuple(p.shape) for p in muon], reverse=True)
    opt = build_optimizer(model, {"name": "muon", "lr": 0.01})
    assert isinstance(opt, SingleDeviceMuonWithAuxAdam)
    x = torch.randint(0, 10, (4,))
    model(x).sum().backward()
    opt.step()
    sd = opt.state_dict()
    kinds = {k for st in sd["state"].values() for k in st}
    assert {"momentum_buffer", "exp_avg", "exp_avg_sq", "step"} <= kinds
    assert all(isinstance(st["step"], int) for st in sd["state"].values() if "step" in st)
    hyper = build_optimizer(model, {"name": "muonh", "lr": 0.01})
    model(x).sum().backward()
    hyper.step()
    assert "hyperball_radii" in hyper.state_dict()


def test_muon_update_shapes():
    g = torch.randn(8, 3, 2, 2)
    m = torch.zeros_like(g)
    u = muon_update(g.clone(), m, beta=0.95)
    assert u.shape == (8, 12)


def test_ema_closed_forms_and_state():
    model = torch.nn.Linear(3, 1, bias=False)
    with torch.no_grad():
        model.weight.fill_(1.0)
    ema = EMA(model, decay=0.9, offload_to_cpu=False)
    with torch.no_grad():
        model.weight.fill_(0.0)
    for _ in range(3):
        ema.update(model)
    assert torch.allclose(ema.shadow["weight"], torch.full((1, 3), 0.9 ** 3))
    thin = EMA(model, decay=0.9, update_every=2, offload_to_cpu=False)
    with torch.no_grad():
        model.weight.fill_(1.0)
    thin.update(model)
    thin.update(model)
    assert torch.allclose(thin.shadow["weight"], torch.full((1, 3), 1 - 0.81))
    st = thin.state_dict()
    assert {"decay", "profile", "gamma", "num_updates", "step_counter", "last_update_step_counter", "update_every",
            "compensate_update_every", "shadow", "dtype"} == set(st)
    power = EMA(model, decay=0.9, profile="power", gamma=6.94, offload_to_cpu=False)
    with torch.no_grad():
        model.weight.fill_(3.0)
    power.update(model)  # the power profile's first update (t = 1) has decay 0: it copies the parameter
    assert torch.equal(power.shadow["weight"], torch.full((1, 3), 3.0))
    with torch.no_grad():
        model.weight.fill_(5.0)
    power.update(model)  # t = 2: decay (1/2) ** (gamma + 1)
    d = 0.5 ** 7.94
    assert torch.allclose(power.shadow["weight"], torch.full((1, 3), 3.0 * d + 5.0 * (1 - d)))
    assert abs(srel_from_gamma(gamma_from_srel(0.1)) - 0.1) < 1e-6
    a, b = ls_coeffs_for_power_profile(100, 5.0, 10.0, 5.0)
    assert abs(a - 1.0) < 1e-6 and abs(b) < 1e-6
