"""Freeze the garbage collector's view after warm-up (reference: koochak/utils/collector.py:18-41).

A full cyclic collection walks every tracked object; with compiled graphs
alive that takes about a second per rank, at different steps on different
ranks, and the others wait in the next collective. After the second update
(and again whenever a new compiled graph appears) everything alive is frozen
out of future collections.
"""

from __future__ import annotations

import gc
import sys

__all__ = ["WARM_UPDATES", "WarmFreeze", "compiled_graphs"]

WARM_UPDATES = 2


def compiled_graphs() -> int:
    utils = sys.modules.get("torch._dynamo.utils")
    return 0 if utils is None else int(utils.counters["stats"]["unique_graphs"])


class WarmFreeze:
    def __init__(self) -> None:
        self.updates = 0
        self.graphs: int | None = None

    def update(self) -> None:
        self.updates += 1
        if self.updates < WARM_UPDATES:
            return
        now = compiled_graphs()
        if now != self.graphs:
            gc.collect()
            gc.freeze()
            self.graphs = now
