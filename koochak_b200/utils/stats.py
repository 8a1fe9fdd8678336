"""Running statistics of scalar series for logs.

(behaviour of reference koochak/utils/stats.py:10-89)

* ``SmoothedMeter``: statistics of the last ``window_size`` values plus the
  weighted mean of everything seen;
* ``Throughput``: items per second across the last ``window_size`` updates;
* ``EMA``: exponential moving average of one scalar (the first value seeds it).
"""

from __future__ import annotations

import statistics
import time
from collections import deque
from typing import Callable, Deque, Iterable, Optional, Tuple

__all__ = ["SmoothedMeter", "Throughput", "EMA"]


def _or_zero(fn: Callable[[Iterable[float]], float], values: Deque[float]) -> float:
    return float(fn(values)) if values else 0.0


class SmoothedMeter:
    """Windowed median / mean / extrema and a global (count-weighted) mean."""

    def __init__(self, window_size: int = 100) -> None:
        self.window_size = int(window_size)
        self.deque: Deque[float] = deque(maxlen=self.window_size)
        self.total = 0.0
        self.count = 0

    def update(self, value: float, n: int = 1) -> None:
        x = float(value)
        self.deque.append(x)
        self.count += n
        self.total += x * n

    median = property(lambda self: _or_zero(statistics.median, self.deque))
    avg = property(lambda self: _or_zero(statistics.fmean, self.deque))
    max = property(lambda self: _or_zero(max, self.deque))
    min = property(lambda self: _or_zero(min, self.deque))

    @property
    def global_avg(self) -> float:
        return self.total / self.count if self.count > 0 else 0.0


class Throughput:
    """Items per second between the oldest and newest of the last ``window_size`` updates."""

    def __init__(self, window_size: int = 50) -> None:
        self._events: Deque[Tuple[float, int]] = deque(maxlen=window_size)

    def update(self, n_items: int) -> None:
        self._events.append((time.time(), int(n_items)))

    @property
    def times(self):
        return [t for t, _ in self._events]

    @property
    def counts(self):
        return [n for _, n in self._events]

    @property
    def it_per_s(self) -> float:
        if len(self._events) < 2:
            return 0.0
        elapsed = self._events[-1][0] - self._events[0][0]
        if elapsed <= 0:
            return 0.0
        return sum(n for _, n in self._events) / elapsed


class EMA:
    """``value <- alpha * value + (1 - alpha) * x``; the first update sets ``value = x``."""

    def __init__(self, alpha: float = 0.98) -> None:
        self.alpha = float(alpha)
        self.value: Optional[float] = None

    def update(self, x: float) -> float:
        x = float(x)
        self.value = x if self.value is None else x + self.alpha * (self.value - x)
        return self.value
