"""Process-group bootstrap and rank queries.

(behaviour of reference koochak/core/dist.py:19-102)

Restart safety: when torchrun's elastic agent hosts the rendezvous store
(``TORCHELASTIC_USE_AGENT_STORE=True``), every attempt of the job builds its
process group on its own key space, ``/koochak/attempt_<restart count>`` of
the agent's TCP store, so workers of a restarted attempt never read keys
that a failed attempt left behind. The prefix is a contract with launchers
and with the reference (both frameworks can share one torchrun agent).
"""

from __future__ import annotations

import datetime
import os
from typing import Any, Dict, Optional

import torch

__all__ = ["is_initialized", "init_process_group", "barrier", "rank", "world_size", "rank0", "print0",
           "torchelastic_attempt_store", "local_rank"]

_ATTEMPT_PREFIX = "/koochak/attempt_{}"


def is_initialized() -> bool:
    try:
        import torch.distributed as td
    except ImportError:  # pragma: no cover
        return False
    return td.is_available() and td.is_initialized()


def torchelastic_attempt_store(timeout: datetime.timedelta) -> Optional["torch.distributed.Store"]:
    """The agent's store seen through this attempt's prefix; ``None`` when torchrun does not host it."""

    if os.environ.get("TORCHELASTIC_USE_AGENT_STORE") != "True":
        return None
    import torch.distributed as td

    agent = td.TCPStore(os.environ["MASTER_ADDR"], int(os.environ["MASTER_PORT"]), is_master=False, timeout=timeout)
    return td.PrefixStore(_ATTEMPT_PREFIX.format(os.environ["TORCHELASTIC_RESTART_COUNT"]), agent)


def _group_kwargs(backend: str, init_method: Optional[str], timeout: Optional[float], rank_: Optional[int],
                  world: Optional[int]) -> Dict[str, Any]:
    kw: Dict[str, Any] = {"backend": backend}
    if timeout is not None:
        kw["timeout"] = datetime.timedelta(seconds=float(timeout))
    env_rendezvous = init_method is None or init_method == "env://"
    store = None
    if env_rendezvous:
        from torch.distributed.constants import default_pg_timeout

        store = torchelastic_attempt_store(kw.get("timeout", default_pg_timeout))
    if store is not None:
        # A store-based group needs explicit rank and size.
        kw["store"] = store
        rank_ = int(os.environ["RANK"]) if rank_ is None else rank_
        world = int(os.environ["WORLD_SIZE"]) if world is None else world
    elif init_method is not None:
        kw["init_method"] = init_method
    for key, value in (("rank", rank_), ("world_size", world)):
        if value is not None:
            kw[key] = int(value)
    return kw


def init_process_group(backend: str = "nccl", init_method: Optional[str] = None, timeout: Optional[float] = None, *,
                       rank: Optional[int] = None, world_size: Optional[int] = None) -> None:
    """Create the default process group once (later calls are no-ops)."""

    import torch.distributed as td

    if not td.is_available():
        raise RuntimeError("torch.distributed not available in this build")
    if not is_initialized():
        td.init_process_group(**_group_kwargs(backend, init_method, timeout, rank, world_size))


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
