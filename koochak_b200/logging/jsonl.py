"""One JSON object per line, keys sorted (reference: koochak/logging/jsonl.py:12-48)."""

from __future__ import annotations

import json
import os
from typing import Any, Dict

from ._sink import sink_hooks

__all__ = ["JSONLLogger", "make_jsonl_hooks"]


class JSONLLogger:
    def __init__(self, path: str) -> None:
        self.path = path
        os.makedirs(os.path.dirname(os.path.abspath(path)) or ".", exist_ok=True)
        self._fh = open(path, "a", encoding="utf-8")

    def write(self, payload: Dict[str, Any]) -> None:
        if self._fh is not None:
            self._fh.write(json.dumps(payload, sort_keys=True, default=str) + "\n")
            self._fh.flush()

    def close(self) -> None:
        if self._fh is not None:
            self._fh.close()
            self._fh = None


def make_jsonl_hooks(path: str):
    lg = JSONLLogger(path)
    return sink_hooks(lg.write, lg.close)
