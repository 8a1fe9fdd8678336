"""Small running statistics (reference: koochak/utils/stats.py:10-89)."""

from __future__ import annotations

import collections
import statistics
import time
from typing import Deque, Optional

__all__ = ["SmoothedMeter", "Throughput", "EMA"]


class SmoothedMeter:
    """Windowed median/mean plus a global mean of a scalar series."""

    def __init__(self, window_size: int = 100) -> None:
        self.window_size = int(window_size)
        self.deque: Deque[float] = collections.deque(maxlen=self.window_size)
        self.total = 0.0
        self.count = 0

    def update(self, value: float, n: int = 1) -> None:
        v = float(value)
        self.deque.append(v)
        self.total += v * n
        self.count += n

    @property
    def median(self) -> float:
        return float(statistics.median(self.deque)) if self.deque else 0.0

    @property
    def avg(self) -> float:
        return sum(self.deque) / len(self.deque) if self.deque else 0.0

    @property
    def global_avg(self) -> float:
        return self.total / max(1, self.count)

    @property
    def max(self) -> float:
        return max(self.deque) if self.deque else 0.0

    @property
    def min(self) -> float:
        return min(self.deque) if self.deque else 0.0


class Throughput:
    """Items per second over a sliding window of timestamps."""

    def __init__(self, window_size: int = 50) -> None:
        self.times: Deque[float] = collections.deque(maxlen=window_size)
        self.counts: Deque[int] = collections.deque(maxlen=window_size)

    def update(self, n_items: int) -> None:
        self.times.append(time.time())
        self.counts.append(int(n_items))

    @property
    def it_per_s(self) -> float:
        if len(self.times) < 2:
            return 0.0
        span = self.times[-1] - self.times[0]
        return sum(self.counts) / span if span > 0 else 0.0


class EMA:
    """Exponential moving average of a scalar: v = a*v + (1-a)*x."""

    def __init__(self, alpha: float = 0.98) -> None:
        self.alpha = float(alpha)
        self.value: Optional[float] = None

    def update(self, x: float) -> float:
        x = float(x)
        self.value = x if self.value is None else self.alpha * self.value + (1.0 - self.alpha) * x
        return self.value
