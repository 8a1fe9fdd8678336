"""Process-group bootstrap from config and launcher environment (reference: koochak/core/launch.py:108-170)."""

from __future__ import annotations

import os
from typing import Any, Dict, Mapping, Optional

import torch

from . import dist as dist_lib

__all__ = ["initialize"]

_LOCAL_RANK_VARS = ("LOCAL_RANK", "MPI_LOCALRANKID", "OMPI_COMM_WORLD_LOCAL_RANK", "MV2_COMM_WORLD_LOCAL_RANK",
                    "SLURM_LOCALID")


def _int_or_none(value: Any, name: str) -> Optional[int]:
    if value is None:
        return None
    try:
        return int(value)
    except (TypeError, ValueError) as exc:
        raise RuntimeError(f"[dist] Expected an integer for {name}, got {value!r}") from exc


def _first_env_int(names) -> Optional[int]:
    for n in names:
        if n in os.environ:
            return _int_or_none(os.environ[n], n)
    return None


def _dist_section(config: Optional[Mapping[str, Any]]) -> Mapping[str, Any]:
    if not isinstance(config, Mapping):
        return {}
    for key in ("dist", "distributed"):
        if isinstance(config.get(key), Mapping):
            return config[key]
    return config


def _backend(cfg: Mapping[str, Any]) -> str:
    b = cfg.get("backend") or os.environ.get("TORCH_DIST_BACKEND")
    return str(b) if b else ("nccl" if torch.cuda.is_available() else "gloo")


def _init_method(cfg: Mapping[str, Any]) -> Optional[str]:
    m = cfg.get("init_method") or os.environ.get("TORCH_DIST_INIT_METHOD")
    if m:
        return str(m)
    return "env://" if (os.environ.get("MASTER_ADDR") or os.environ.get("MASTER_PORT")) else None


def _timeout(cfg: Mapping[str, Any]) -> Optional[float]:
    t = cfg.get("timeout") or os.environ.get("TORCH_DIST_TIMEOUT")
    if t is None:
        return None
    try:
        return float(t)
    except (TypeError, ValueError) as exc:
        raise RuntimeError(f"[dist] Invalid timeout value: {t!r}") from exc


def _set_device(local_rank: Optional[int]) -> Optional[int]:
    if not torch.cuda.is_available():
        return None
    n = torch.cuda.device_count()
    if local_rank is not None:
        if not 0 <= local_rank < n:
            raise RuntimeError(f"[dist] local_rank={local_rank} is out of range for {n} CUDA devices")
        torch.cuda.set_device(local_rank)
        return local_rank
    try:
        cur = torch.cuda.current_device()
    except RuntimeError:
        cur = 0
    torch.cuda.set_device(cur)
    return int(cur)


def initialize(config: Optional[Mapping[str, Any]] = None) -> Dict[str, Any]:
    """Initialise the process group when the launcher or config asks for one.

    Returns ``{rank, world_size, is_rank0, device}``.
    """

    cfg = _dist_section(config)
    rank = _int_or_none(cfg.get("rank"), "rank") or _first_env_int(("RANK", "SLURM_PROCID"))
    world = _int_or_none(cfg.get("world_size"), "world_size") or _first_env_int(("WORLD_SIZE", "SLURM_NTASKS"))
    local = _int_or_none(cfg.get("local_rank"), "local_rank") or _first_env_int(_LOCAL_RANK_VARS)
    device = _set_device(local)
    if dist_lib.is_initialized():
        rank, world = dist_lib.rank(), dist_lib.world_size()
    else:
        wanted = any([os.environ.get("MASTER_ADDR"), os.environ.get("MASTER_PORT"), rank is not None,
                      world is not None])
        if wanted and not torch.distributed.is_available():
            raise RuntimeError("[dist] torch.distributed requested but not available in this build")
        if wanted:
            backend, method = _backend(cfg), _init_method(cfg)
            try:
                dist_lib.init_process_group(backend=backend, init_method=method, timeout=_timeout(cfg), rank=rank,
                                            world_size=world)
            except Exception as exc:
                raise RuntimeError(f"[dist] Failed to initialize process group (backend={backend}, "
                                   f"init_method={method or 'default'}, rank={rank}, world_size={world})") from exc
            rank, world = dist_lib.rank(), dist_lib.world_size()
    rank = 0 if rank is None else int(rank)
    world = 1 if world is None else int(world)
    return {"rank": rank, "world_size": world, "is_rank0": rank == 0, "device": device}
