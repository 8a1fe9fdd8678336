"""Append-only CSV metrics (reference: koochak/logging/csv.py:13-80).

The column set is fixed by the first row written (``step`` first, the other
keys sorted) unless given; keys that appear later are dropped with one
warning per key, so schema drift is visible rather than silent.
"""

from __future__ import annotations

import csv as _csv
import os
import warnings
from typing import Any, Dict, List, Optional, Set

from ._sink import sink_hooks

__all__ = ["CSVLogger", "make_csv_hooks"]


class CSVLogger:
    def __init__(self, path: str, fieldnames: Optional[List[str]] = None) -> None:
        self.path = path
        os.makedirs(os.path.dirname(os.path.abspath(path)) or ".", exist_ok=True)
        self.fieldnames = list(fieldnames) if fieldnames else None
        self._fh = None
        self._writer = None
        self._warned: Set[str] = set()

    def _open(self, keys: List[str]) -> None:
        if self.fieldnames is None:
            self.fieldnames = ["step"] + sorted(k for k in keys if k != "step")
        fresh = not os.path.exists(self.path)
        self._fh = open(self.path, "a", newline="", encoding="utf-8")
        self._writer = _csv.DictWriter(self._fh, fieldnames=self.fieldnames)
        if fresh:
            self._writer.writeheader()

    def write(self, payload: Dict[str, Any]) -> None:
        if self._writer is None:
            self._open(list(payload))
        cols = set(self.fieldnames or ())
        dropped = [k for k in payload if k not in cols and k not in self._warned]
        if dropped:
            warnings.warn(f"CSVLogger: dropping keys not in initial schema: {sorted(dropped)}", UserWarning)
            self._warned.update(dropped)
        self._writer.writerow({k: payload.get(k) for k in self.fieldnames})
        self._fh.flush()

    def close(self) -> None:
        if self._fh is not None:
            self._fh.close()
        self._fh = self._writer = None


def make_csv_hooks(path: str):
    lg = CSVLogger(path)
    return sink_hooks(lg.write, lg.close)
