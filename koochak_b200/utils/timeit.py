"""Wall-clock and CUDA-event timers (reference: koochak/utils/timeit.py:10-37).

``Timer``/``time_block`` are host wall-clock; ``CudaTimer`` brackets a region
with CUDA events on the current stream and reports device milliseconds.
"""

from __future__ import annotations

import time
from contextlib import contextmanager
from typing import Dict, Iterator, Optional

__all__ = ["Timer", "time_block", "CudaTimer"]


class Timer:
    """``with Timer() as t: ...`` then ``t.elapsed`` (seconds)."""

    def __enter__(self) -> "Timer":
        self._t0 = time.perf_counter()
        self.elapsed = 0.0
        return self

    def __exit__(self, *exc) -> bool:
        self.elapsed = time.perf_counter() - self._t0
        return False


@contextmanager
def time_block(store: Dict[str, float], key: str) -> Iterator[None]:
    """Add the elapsed wall time of the block to ``store[key]``."""

    t0 = time.perf_counter()
    try:
        yield None
    finally:
        store[key] = store.get(key, 0.0) + (time.perf_counter() - t0)


class CudaTimer:
    """Device-side timing of a region with CUDA events (milliseconds)."""

    def __init__(self, stream=None) -> None:
        import torch

        self._torch = torch
        self.stream = stream
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)
        self.elapsed_ms: Optional[float] = None

    def __enter__(self) -> "CudaTimer":
        self.start.record(self.stream)
        return self

    def __exit__(self, *exc) -> bool:
        self.end.record(self.stream)
        return False

    def result(self) -> float:
        self.end.synchronize()
        self.elapsed_ms = float(self.start.elapsed_time(self.end))
        return self.elapsed_ms
