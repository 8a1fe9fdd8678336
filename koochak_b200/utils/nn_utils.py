"""Parameter tags and Muon/Adam group construction (reference: koochak/utils/nn_utils.py:8-95).

Tags: ``wd`` (receives weight decay) and ``mapping`` (never Muon, even when
2-D and decayed). The Muon group is sorted by size, largest first; that order
defines optimizer-state indices in checkpoints.
"""

from __future__ import annotations

from typing import Any

import torch.nn as nn

__all__ = ["tag_param", "tag_module", "apply_wd", "prepare_param_groups_for_muon", "has_tag"]


def tag_param(param: nn.Parameter, tag: str) -> nn.Parameter:
    tags = getattr(param, "_tags", None)
    if tags is None:
        param._tags = {tag}  # type: ignore[attr-defined]
    else:
        tags.add(tag)
    return param


def tag_module(module: nn.Module, tag: str) -> nn.Module:
    for p in module.parameters():
        tag_param(p, tag)
    return module


def apply_wd(module: nn.Module) -> nn.Module:
    """Tag every parameter whose name ends in ``weight`` with ``wd``."""

    for name, p in module.named_parameters():
        if name.endswith("weight"):
            tag_param(p, "wd")
    return module


def has_tag(param: nn.Parameter, tag: str) -> bool:
    return tag in getattr(param, "_tags", set())


def prepare_param_groups_for_muon(model: nn.Module, lr: float, weight_decay: float) -> list[dict[str, Any]]:
    """Groups in this order: Adam without decay, Adam with decay, Muon."""

    muon, adam_wd, adam_nowd = [], [], []
    for _, p in model.named_parameters():
        if not p.requires_grad:
            continue
        decayed = has_tag(p, "wd")
        if p.ndim >= 2 and decayed and not has_tag(p, "mapping"):
            muon.append(p)
        elif decayed:
            adam_wd.append(p)
        else:
            adam_nowd.append(p)

    def adam_group(params, wd):
        return {"params": params, "betas": (0.9, 0.95), "eps": 1e-10, "lr": float(lr), "weight_decay": float(wd),
                "use_muon": False}

    groups: list[dict[str, Any]] = []
    if adam_nowd:
        groups.append(adam_group(adam_nowd, 0.0))
    if adam_wd:
        groups.append(adam_group(adam_wd, weight_decay))
    if muon:
        groups.append({"params": sorted(muon, key=lambda t: t.size(), reverse=True), "lr": float(lr),
                       "weight_decay": float(weight_decay), "momentum": 0.95, "use_muon": True})
    return groups
