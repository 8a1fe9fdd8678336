"""Optimizer and scheduler factories from config (reference: koochak/optim/build.py:52-243).

Names: ``adamw`` (on CUDA fp32 parameters the native multi-tensor
``FusedAdamW``, elsewhere ``torch.optim.AdamW``), ``adam`` / ``sgd`` (PyTorch
optimizers), ``muon`` / ``normuon`` and the Hyperball
variants ``muonh`` / ``normuonh`` (aliases ``hyperball-muon`` ...). Muon
needs the model (or param groups with ``use_muon``); the distributed class is
chosen iff a process group is initialised. Schedulers: ``cosine``,
``cosine_warmup``, ``linear_warmup``, ``step``, ``plateau``.
"""

from __future__ import annotations

from typing import Any, Mapping, Optional

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.optim import SGD, Adam, AdamW, Optimizer
from torch.optim.lr_scheduler import CosineAnnealingLR, LambdaLR, ReduceLROnPlateau, SequentialLR, StepLR, _LRScheduler

from ..utils.nn_utils import prepare_param_groups_for_muon
from .muon import FusedAdamW, HyperballOptimizer, MuonWithAuxAdam, NorMuonWithAuxAdam, SingleDeviceMuonWithAuxAdam, \
    SingleDeviceNorMuonWithAuxAdam

__all__ = ["build_optimizer", "build_scheduler"]

_HYPERBALL = {"muonh": "muon", "hyperball-muon": "muon", "hyperball_muon": "muon", "hyperballmuon": "muon",
              "normuonh": "normuon", "hyperball-normuon": "normuon", "hyperball_normuon": "normuon",
              "hyperballnormuon": "normuon"}
_MUON_FAMILY = {"muon", "normuon"} | set(_HYPERBALL)


def _bool_or_none(v: Any) -> Optional[bool]:
    if v is None or isinstance(v, bool):
        return v
    if isinstance(v, str):
        s = v.strip().lower()
        if s in {"1", "true", "yes", "on"}:
            return True
        if s in {"0", "false", "no", "off"}:
            return False
    return bool(v)


def _params_of(params):
    return params.parameters() if isinstance(params, nn.Module) else params


def _dist_on() -> bool:
    return dist.is_available() and dist.is_initialized()


def _build_muon(params, *, name: str, lr: float, weight_decay: float, muon_lr: Optional[float],
                adam_lr: Optional[float], foreach_adam_update: Optional[bool], hyperball_eps: float,
                hyperball_radius_scale: float, hyperball_projection: str) -> Optimizer:
    hyper = name in _HYPERBALL
    base = _HYPERBALL.get(name, name)
    single_cls, dist_cls = ((SingleDeviceMuonWithAuxAdam, MuonWithAuxAdam) if base == "muon"
                            else (SingleDeviceNorMuonWithAuxAdam, NorMuonWithAuxAdam))
    if isinstance(params, nn.Module):
        groups = prepare_param_groups_for_muon(params, lr=lr, weight_decay=weight_decay)
    elif isinstance(params, (list, tuple)) and params and isinstance(params[0], dict):
        groups = list(params)
    else:
        raise ValueError("For optimizer=name: 'Muon', 'MuonH', 'NorMuon', 'NorMuonH', 'hyperball-muon', or "
                         "'hyperball-normuon', pass the model module or a list of param_groups with 'use_muon' flags.")
    for g in groups:
        if g.get("use_muon", False):
            if muon_lr is not None:
                g["lr"] = muon_lr
        elif adam_lr is not None:
            g["lr"] = adam_lr
    if foreach_adam_update is not None:
        groups = [g if g.get("use_muon", False) else dict(g, foreach_adam_update=foreach_adam_update) for g in groups]
    matrices = [p for g in groups if g.get("use_muon", False) for p in g.get("params", [])]
    if hyper:
        # Projection back to the initial radius makes decoupled decay redundant.
        groups = [dict(g, weight_decay=0.0) for g in groups]
    inner = (dist_cls if _dist_on() else single_cls)(groups)
    if not hyper:
        return inner
    return HyperballOptimizer(inner, matrices, eps=float(hyperball_eps), radius_scale=float(hyperball_radius_scale),
                              projection=str(hyperball_projection))


def _native_adamw_ok(plist) -> bool:
    tensors = [p for p in plist if isinstance(p, torch.Tensor)]
    if not tensors or len(tensors) != len(plist):
        return False
    if not all(p.is_cuda and p.dtype == torch.float32 for p in tensors):
        return False
    from ..ops._ext import available

    return available()


def build_optimizer(params, cfg: Optional[Mapping[str, Any]]) -> Optimizer:
    cfg = cfg or {}
    name = str(cfg.get("name", "adamw")).lower()
    lr = float(cfg.get("lr", 3e-4))
    wd = float(cfg.get("weight_decay", 0.0))
    if name in ("adamw", "adam"):
        betas = tuple(cfg.get("betas", (0.9, 0.999)))
        eps = float(cfg.get("eps", 1e-8))
        plist = list(_params_of(params))
        if name == "adamw" and _native_adamw_ok(plist):
            return FusedAdamW(plist, lr=lr, betas=betas, eps=eps, weight_decay=wd)
        cls = AdamW if name == "adamw" else Adam
        return cls(plist, lr=lr, betas=betas, eps=eps, weight_decay=wd)
    if name == "sgd":
        return SGD(_params_of(params), lr=lr, momentum=float(cfg.get("momentum", 0.9)), weight_decay=wd,
                   nesterov=bool(cfg.get("nesterov", False)))
    if name in _MUON_FAMILY:
        raw_m, raw_a = cfg.get("muon_lr"), cfg.get("adam_lr")
        return _build_muon(params, name=name, lr=lr, weight_decay=wd,
                           muon_lr=float(raw_m) if raw_m is not None else None,
                           adam_lr=float(raw_a) if raw_a is not None else None,
                           foreach_adam_update=_bool_or_none(cfg.get("foreach_adam_update")),
                           hyperball_eps=float(cfg.get("hyperball_eps", 1.0e-8)),
                           hyperball_radius_scale=float(cfg.get("hyperball_radius_scale", 1.0)),
                           hyperball_projection=str(cfg.get("hyperball_projection", "sphere")))
    raise ValueError(f"Unsupported optimizer name: {name}")


def build_scheduler(optimizer: Optimizer, cfg: Optional[Mapping[str, Any]],
                    train_cfg: Mapping[str, Any]) -> Optional[_LRScheduler]:
    if not cfg:
        return None
    name = str(cfg.get("name", "none")).lower()
    if name in ("none", "never", "off"):
        return None
    total = int(cfg.get("T_max") or cfg.get("t_max") or train_cfg.get("max_steps", 1000))
    if name == "cosine":
        return CosineAnnealingLR(optimizer, T_max=total, eta_min=float(cfg.get("eta_min", 0.0)))
    if name in ("cosine_warmup", "warmup_cosine", "cosinewithwarmup"):
        warm = int(cfg.get("warmup_steps", 0))
        cosine = CosineAnnealingLR(optimizer, T_max=max(1, total - warm), eta_min=float(cfg.get("eta_min", 0.0)))
        if warm <= 0:
            return cosine
        ramp = LambdaLR(optimizer, lr_lambda=lambda s: s / warm)
        return SequentialLR(optimizer, [ramp, cosine], milestones=[warm])
    if name in ("linear_warmup", "warmup_constant", "constant_warmup"):
        warm = max(1, int(cfg.get("warmup_steps", 0)))
        return LambdaLR(optimizer, lr_lambda=lambda s: min(1.0, max(0.0, float(s)) / float(warm)))
    if name == "step":
        return StepLR(optimizer, step_size=int(cfg.get("step_size", 1000)), gamma=float(cfg.get("gamma", 0.1)))
    if name == "plateau":
        return ReduceLROnPlateau(optimizer, mode=str(cfg.get("mode", "min")), factor=float(cfg.get("factor", 0.1)),
                                 patience=int(cfg.get("patience", 10)))
    raise ValueError(f"Unsupported scheduler name: {name}")
