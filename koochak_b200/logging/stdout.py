"""Tab-separated step lines on stdout (reference: koochak/logging/stdout.py:44-102).

A line is ``step<TAB>N<TAB>key<TAB>value...``: ``loss`` and ``lr`` first, then
the remaining keys in sorted order; floats use 4 significant digits, bools
print as 1/0 and long strings are cut to 64 characters.
"""

from __future__ import annotations

import json
import sys
from typing import Any, Dict, List

from ..core.hooks import rank0_only
from ._sink import eval_payload, is_bad_float, scalar

__all__ = ["StdoutLogger", "make_stdout_hooks", "log_step_tsv"]

_FIRST = ("loss", "lr")


def _text(v: Any) -> str:
    v = scalar(v)
    if isinstance(v, bool):
        return "1" if v else "0"
    if isinstance(v, int):
        return str(v)
    if isinstance(v, float):
        return str(v) if is_bad_float(v) else f"{v:.4g}"
    s = str(v)
    return s if len(s) <= 64 else s[:61] + "..."


def log_step_tsv(payload: Dict[str, Any], *, file=None) -> None:
    out = file if file is not None else sys.stdout
    fields: List[str] = []
    if payload.get("step") is not None:
        fields += ["step", _text(payload["step"])]
    keys = [k for k in _FIRST if k in payload]
    keys += sorted(k for k in payload if k != "step" and k not in _FIRST)
    for k in keys:
        fields += [k, _text(payload[k])]
    print("\t".join(fields), file=out, flush=True)


class StdoutLogger:
    def __init__(self, file=None) -> None:
        self.file = file if file is not None else sys.stdout

    def on_log(self, logs: Dict[str, Any], ctx: Dict[str, Any]) -> None:
        log_step_tsv(logs, file=self.file)

    def on_eval_end(self, metrics: Dict[str, Any], ctx: Dict[str, Any]) -> None:
        log_step_tsv(eval_payload(metrics, ctx), file=self.file)

    def on_train_start(self, ctx: Dict[str, Any]) -> None:
        print(f"[koochak] device={ctx.get('device')} rank={ctx.get('rank')}/{ctx.get('world_size')}",
              file=self.file, flush=True)
        if ctx.get("config_json") is not None:
            print("[config] " + json.dumps(ctx["config_json"], sort_keys=True, default=str), file=self.file,
                  flush=True)

    def on_train_end(self, ctx: Dict[str, Any]) -> None:
        print("[koochak] training finished", file=self.file, flush=True)


def make_stdout_hooks(file=None) -> Dict[str, List]:
    lg = StdoutLogger(file)
    return {ev: [rank0_only(getattr(lg, ev))] for ev in ("on_train_start", "on_log", "on_eval_end", "on_train_end")}
