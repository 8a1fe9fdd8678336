"""Random-number state: capture, restore and seeding of every generator a run uses.

(behaviour of reference koochak/utils/seed.py:16-61)

Each generator family is one ``_Source`` entry (its checkpoint key, how to
read its state, how to restore it, how to seed it), so capture, restore and
seeding are the same loop over one table. The keys ``python``, ``numpy``,
``torch_cpu`` and ``torch_cuda`` are part of the checkpoint format: a source
that is unavailable (no numpy, no CUDA) is recorded as ``None`` and skipped
on restore.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Callable, Dict, Optional

import torch

try:
    import numpy as _np
except ImportError:  # pragma: no cover
    _np = None  # type: ignore[assignment]

__all__ = ["get_rng_state", "set_rng_state", "set_all_seeds", "make_worker_init_fn"]


@dataclass(frozen=True)
class _Source:
    key: str
    available: Callable[[], bool]
    capture: Callable[[], Any]
    restore: Callable[[Any], None]
    seed: Callable[[int], None]


def _always() -> bool:
    return True


_SOURCES = (
    _Source("numpy", lambda: _np is not None, lambda: _np.random.get_state(), lambda s: _np.random.set_state(s),
            lambda n: _np.random.seed(n)),
    _Source("python", _always, random.getstate, random.setstate, random.seed),
    _Source("torch_cpu", _always, torch.get_rng_state, torch.set_rng_state, torch.manual_seed),
    _Source("torch_cuda", torch.cuda.is_available, torch.cuda.get_rng_state_all, torch.cuda.set_rng_state_all,
            torch.cuda.manual_seed_all),
)


def get_rng_state() -> Dict[str, Any]:
    """State of every generator, keyed as in checkpoints (``None`` for an unavailable one)."""

    return {src.key: (src.capture() if src.available() else None) for src in _SOURCES}


def set_rng_state(state: Dict[str, Any]) -> None:
    """Restore what ``get_rng_state`` captured; missing or ``None`` entries are left alone."""

    for src in _SOURCES:
        value: Optional[Any] = state.get(src.key)
        if value is not None and src.available():
            src.restore(value)


def _seed_everything(seed: int, keys=None) -> None:
    for src in _SOURCES:
        if (keys is None or src.key in keys) and src.available():
            src.seed(seed)


def set_all_seeds(seed: int) -> None:
    """Seed python, numpy, torch CPU and all CUDA generators; deterministic algorithms stay off."""

    _seed_everything(int(seed))
    torch.use_deterministic_algorithms(False)


def make_worker_init_fn(base_seed: int, *, rank: int = 0, worker_seed_offset: int = 1000):
    """A DataLoader ``worker_init_fn``: worker ``w`` of rank ``r`` is seeded with ``base + r * offset + w``.

    Only the host generators are seeded (python, numpy, torch CPU); workers do not touch CUDA.
    """

    origin = int(base_seed) + int(rank) * int(worker_seed_offset)

    def init(worker_id: int) -> None:
        _seed_everything(origin + int(worker_id), keys=("python", "numpy", "torch_cpu"))

    return init
