"""Process-group helpers that survive torchrun restarts (reference: koochak/core/dist.py:19-102).

Under torchrun's agent store (``TORCHELASTIC_USE_AGENT_STORE=True``) the
process group is created on a per-attempt ``PrefixStore`` so that workers of a
restarted attempt can never read the previous attempt's rendezvous keys.
"""

from __future__ import annotations

import datetime
import os
from typing import Optional

import torch

__all__ = ["is_initialized", "init_process_group", "barrier", "rank", "world_size", "rank0", "print0",
           "torchelastic_attempt_store", "local_rank"]


def is_initialized() -> bool:
    try:
        return torch.distributed.is_available() and torch.distributed.is_initialized()
    except ImportError:
        return False


def torchelastic_attempt_store(timeout: datetime.timedelta) -> Optional["torch.distributed.Store"]:
    """torchrun's worker store under ``/koochak/attempt_<restart count>``, or None outside torchrun."""

    if os.environ.get("TORCHELASTIC_USE_AGENT_STORE") != "True":
        return None
    base = torch.distributed.TCPStore(os.environ["MASTER_ADDR"], int(os.environ["MASTER_PORT"]), is_master=False,
                                      timeout=timeout)
    prefix = f"/koochak/attempt_{os.environ['TORCHELASTIC_RESTART_COUNT']}"
    return torch.distributed.PrefixStore(prefix, base)


def init_process_group(backend: str = "nccl", init_method: Optional[str] = None, timeout: Optional[float] = None, *,
                       rank: Optional[int] = None, world_size: Optional[int] = None) -> None:
    if not torch.distributed.is_available():
        raise RuntimeError("torch.distributed not available in this build")
    if is_initialized():
        return
    kwargs: dict = {"backend": backend}
    if timeout is not None:
        kwargs["timeout"] = datetime.timedelta(seconds=float(timeout))
    store = None
    if init_method in (None, "env://"):
        from torch.distributed.constants import default_pg_timeout

        store = torchelastic_attempt_store(kwargs.get("timeout", default_pg_timeout))
    if store is not None:
        kwargs["store"] = store
        rank = int(os.environ["RANK"]) if rank is None else rank
        world_size = int(os.environ["WORLD_SIZE"]) if world_size is None else world_size
    elif init_method is not None:
        kwargs["init_method"] = init_method
    if rank is not None:
        kwargs["rank"] = int(rank)
    if world_size is not None:
        kwargs["world_size"] = int(world_size)
    torch.distributed.init_process_group(**kwargs)


def barrier() -> None:
    if is_initialized():
        torch.distributed.barrier()


def rank() -> int:
    return torch.distributed.get_rank() if is_initialized() else 0


def world_size() -> int:
    return torch.distributed.get_world_size() if is_initialized() else 1


def rank0() -> bool:
    return rank() == 0


def local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", "0"))


def print0(string: str) -> None:
    if rank0():
        print(string)
