"""Device selection helpers (reference: koochak/utils/device.py:12-71)."""

from __future__ import annotations

import os
from typing import Any, Mapping

import torch
import torch.distributed as dist

__all__ = ["get_device", "ensure_process_device", "get_lr"]

_LOCAL_RANK_VARS = ("LOCAL_RANK", "MPI_LOCALRANKID", "OMPI_COMM_WORLD_LOCAL_RANK", "MV2_COMM_WORLD_LOCAL_RANK")


def get_device(cfg: Mapping[str, Any] | Any) -> torch.device:
    """``cfg.device`` if set, else ``cuda`` when available, else ``cpu``."""

    dev = cfg.get("device") if isinstance(cfg, Mapping) else getattr(cfg, "device", None)
    if dev is None:
        dev = "cuda" if torch.cuda.is_available() else "cpu"
    return torch.device(dev)


def _local_rank(default: int = 0) -> int:
    for var in _LOCAL_RANK_VARS:
        raw = os.environ.get(var)
        if raw is None:
            continue
        try:
            return int(raw)
        except ValueError:
            continue
    if torch.cuda.is_available() and dist.is_available() and dist.is_initialized():
        return dist.get_rank() % max(1, torch.cuda.device_count())
    return default


def ensure_process_device(device: torch.device) -> torch.device:
    """Bind an index-less CUDA device to this process's local rank and make it current."""

    if device.type != "cuda":
        return device
    if device.index is None:
        device = torch.device("cuda", _local_rank())
    torch.cuda.set_device(device)
    return device


def get_lr(optimizer) -> float:
    groups = getattr(optimizer, "param_groups", None) or []
    return float(groups[0].get("lr", 0.0)) if groups else 0.0
