"""Post-hoc power-EMA reconstruction (EDM2, Karras et al. 2024, section 3.2).

(reference: koochak/utils/ema_posthoc.py:52-234)

A power-EMA with exponent g seen at step t weights the history with the
normalised kernel  w_g,t(tau) = (g+1) tau^g / t^(g+1)  on [0, t]. A target
profile (gamma_target, at step T) is approximated by a linear combination of
saved snapshots; the least-squares coefficients solve  G c = j  with
G_ij = <w_i, w_j> and j_i = <w_i, w_target>, where
<w_{g1,t1}, w_{g2,t2}> = (g1+1)(g2+1) min(t1,t2)^(g1+g2+1) / ((g1+g2+1) t1^(g1+1) t2^(g2+1)).
"""

from __future__ import annotations

import math
from typing import Dict, List, Mapping, Optional, Sequence, Tuple

import torch

__all__ = ["ls_coeffs_for_power_profile", "ls_coeffs_for_power_snapshots", "reconstruct_power_ema_state_dict",
           "reconstruct_dual_power_ema_state_dict", "gamma_from_srel", "srel_from_gamma"]


def _inner(g1: float, t1: float, g2: float, t2: float) -> float:
    t1, t2 = max(1.0, float(t1)), max(1.0, float(t2))
    overlap = min(t1, t2)
    return ((g1 + 1.0) * (g2 + 1.0) * overlap ** (g1 + g2 + 1.0)
            / ((g1 + g2 + 1.0) * t1 ** (g1 + 1.0) * t2 ** (g2 + 1.0)))


def srel_from_gamma(gamma: float) -> float:
    g = float(gamma)
    return math.sqrt(g + 1.0) / ((g + 2.0) * math.sqrt(g + 3.0))


def gamma_from_srel(srel: float) -> float:
    """Invert srel(gamma) (monotonically decreasing) by bisection in log space."""

    target = max(1e-9, float(srel))
    lo, hi = 1e-6, 1e6
    for _ in range(64):
        mid = math.sqrt(lo * hi)
        if srel_from_gamma(mid) > target:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def _profile_step(state: Mapping[str, object]) -> float:
    """Model step at which a snapshot's power profile is evaluated."""

    try:
        every = max(1, int(state.get("update_every", 1)))  # type: ignore[arg-type]
    except (TypeError, ValueError):
        every = 1
    if every > 1 or bool(state.get("compensate_update_every", False)):
        raw = state.get("last_update_step_counter", state.get("step_counter", state.get("num_updates", 0)))
    else:
        raw = state.get("num_updates", state.get("step_counter", 0))
    try:
        return max(1.0, float(raw))  # type: ignore[arg-type]
    except (TypeError, ValueError):
        return 1.0


def ls_coeffs_for_power_profile(t: float, gamma1: float, gamma2: float, gamma_target: float) -> Tuple[float, float]:
    """Two-snapshot fit at a common step ``t`` (closed-form 2x2 solve)."""

    t = max(1.0, float(t))
    g11, g22, g12 = _inner(gamma1, t, gamma1, t), _inner(gamma2, t, gamma2, t), _inner(gamma1, t, gamma2, t)
    j1, j2 = _inner(gamma1, t, gamma_target, t), _inner(gamma2, t, gamma_target, t)
    det = g11 * g22 - g12 * g12
    if abs(det) < 1e-20:
        return 1.0, 0.0
    return float((g22 * j1 - g12 * j2) / det), float((g11 * j2 - g12 * j1) / det)


def ls_coeffs_for_power_snapshots(ema_states: Sequence[Mapping[str, object]], *, gamma_target: float,
                                  step: Optional[float] = None) -> List[float]:
    states = list(ema_states)
    if not states:
        raise ValueError("ema_states must contain at least one EMA snapshot")
    for i, s in enumerate(states):
        if str(s.get("profile", "power")).lower() != "power":
            raise ValueError(f"EMA snapshot #{i} must have profile='power'")
        if s.get("gamma") is None:
            raise ValueError(f"EMA snapshot #{i} is missing gamma")
    gammas = [float(s["gamma"]) for s in states]  # type: ignore[arg-type]
    steps = [_profile_step(s) for s in states]
    t_target = max(1.0, float(step)) if step is not None else max(steps)
    n = len(states)
    gram = torch.tensor([[_inner(gammas[i], steps[i], gammas[j], steps[j]) for j in range(n)] for i in range(n)],
                        dtype=torch.float64)
    rhs = torch.tensor([_inner(gammas[i], steps[i], float(gamma_target), t_target) for i in range(n)],
                       dtype=torch.float64)
    try:
        coef = torch.linalg.solve(gram, rhs)
    except RuntimeError:
        coef = torch.linalg.pinv(gram) @ rhs
    return [float(c) for c in coef]


def _combine(shadows: Sequence[Mapping[str, torch.Tensor]], coeffs: Sequence[float]) -> Dict[str, torch.Tensor]:
    keys = set(shadows[0].keys())
    for s in shadows[1:]:
        keys &= set(s.keys())
    out: Dict[str, torch.Tensor] = {}
    for k in sorted(keys):
        ref = shadows[0][k]
        if not isinstance(ref, torch.Tensor):
            continue
        acc = torch.zeros_like(ref, dtype=torch.float32)
        for c, s in zip(coeffs, shadows):
            v = s[k]
            if not isinstance(v, torch.Tensor):
                raise ValueError(f"EMA shadow value for {k!r} is not a tensor")
            acc.add_(v.to(torch.float32), alpha=float(c))
        out[k] = acc.to(dtype=ref.dtype, device=ref.device)
    return out


def reconstruct_power_ema_state_dict(ema_states: Sequence[Mapping[str, object]], *, step: Optional[float] = None,
                                     gamma_target: Optional[float] = None,
                                     srel_target: Optional[float] = None) -> Dict[str, torch.Tensor]:
    states = list(ema_states)
    if not states:
        raise ValueError("ema_states must contain at least one EMA snapshot")
    if gamma_target is None:
        if srel_target is None:
            raise ValueError("Provide gamma_target or srel_target")
        gamma_target = gamma_from_srel(float(srel_target))
    coeffs = ls_coeffs_for_power_snapshots(states, gamma_target=float(gamma_target), step=step)
    shadows = []
    for i, s in enumerate(states):
        sh = s.get("shadow", {})
        if not isinstance(sh, Mapping):
            raise ValueError(f"EMA snapshot #{i} is missing a shadow mapping")
        shadows.append(sh)
    return _combine(shadows, coeffs)


def reconstruct_dual_power_ema_state_dict(ema_dual_list: List[Dict[str, object]], *, step: int,
                                          gamma_target: Optional[float] = None,
                                          srel_target: Optional[float] = None) -> Dict[str, torch.Tensor]:
    if len(ema_dual_list) < 2:
        raise ValueError("ema_dual_list must contain two EMA snapshots")
    a, b = ema_dual_list[0], ema_dual_list[1]
    if str(a.get("profile", "power")).lower() != "power" or str(b.get("profile", "power")).lower() != "power":
        raise ValueError("Both EMA snapshots must have profile='power'")
    if gamma_target is None:
        if srel_target is None:
            raise ValueError("Provide gamma_target or srel_target")
        gamma_target = gamma_from_srel(float(srel_target))
    w1, w2 = ls_coeffs_for_power_profile(step, float(a.get("gamma")), float(b.get("gamma")), float(gamma_target))
    return _combine([a.get("shadow", {}), b.get("shadow", {})], [w1, w2])  # type: ignore[list-item]
