"""Which device a process computes on.

(behaviour of reference koochak/utils/device.py:12-71)

``get_device`` reads an explicit ``device`` from a config (mapping or
attribute), falling back to CUDA when present. ``ensure_process_device``
turns a bare ``cuda`` into this process's GPU: the first launcher variable
that names a local rank (torchrun, MPICH, Open MPI, MVAPICH), else the
global rank modulo the visible GPUs once a process group exists.
"""

from __future__ import annotations

import os
from typing import Any, Mapping, Optional

import torch
import torch.distributed as dist

__all__ = ["get_device", "ensure_process_device", "get_lr"]

_LAUNCHER_LOCAL_RANK = ("LOCAL_RANK", "MPI_LOCALRANKID", "OMPI_COMM_WORLD_LOCAL_RANK", "MV2_COMM_WORLD_LOCAL_RANK")


def _configured(cfg: Any) -> Optional[str]:
    if isinstance(cfg, Mapping):
        return cfg.get("device")
    return getattr(cfg, "device", None)


def get_device(cfg: Mapping[str, Any] | Any) -> torch.device:
    """``cfg.device`` when set, else ``cuda`` if a GPU is visible, else ``cpu``."""

    name = _configured(cfg)
    return torch.device(name if name is not None else ("cuda" if torch.cuda.is_available() else "cpu"))


def _int_env(var: str) -> Optional[int]:
    try:
        return int(os.environ[var])
    except (KeyError, ValueError):
        return None


def local_rank(default: int = 0) -> int:
    """This process's index among the processes of its node."""

    found = [v for v in (_int_env(var) for var in _LAUNCHER_LOCAL_RANK) if v is not None]
    if found:
        return found[0]
    if torch.cuda.is_available() and dist.is_available() and dist.is_initialized():
        return dist.get_rank() % max(1, torch.cuda.device_count())
    return default


def ensure_process_device(device: torch.device) -> torch.device:
    """Pin an index-less CUDA device to this process's GPU and make it current; other devices pass through."""

    if device.type == "cuda":
        if device.index is None:
            device = torch.device("cuda", local_rank())
        torch.cuda.set_device(device)
    return device


def get_lr(optimizer) -> float:
    """Learning rate of the first parameter group (0.0 without groups)."""

    for group in getattr(optimizer, "param_groups", None) or []:
        return float(group.get("lr", 0.0))
    return 0.0
