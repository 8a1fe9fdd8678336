"""Shared plumbing for the file and stream sinks."""

from __future__ import annotations

import math
from typing import Any, Callable, Dict, List

from ..core.hooks import rank0_only


def scalar(x: Any) -> Any:
    """A tensor becomes a Python number (its mean when it has several elements)."""

    if hasattr(x, "detach") and hasattr(x, "numel"):
        return x.item() if x.numel() == 1 else x.detach().float().mean().item()
    return x


def eval_payload(metrics: Dict[str, Any], ctx: Dict[str, Any]) -> Dict[str, Any]:
    return {"step": ctx.get("step"), **metrics}


def sink_hooks(write: Callable[[Dict[str, Any]], None], close: Callable[[], None]) -> Dict[str, List[Callable]]:
    """Hooks that send train logs and eval metrics to ``write`` on rank 0 and close on exit."""

    def on_log(logs, ctx):
        write(logs)

    def on_eval_end(metrics, ctx):
        write(eval_payload(metrics, ctx))

    def on_close(*_a, **_k):
        close()

    return {
        "on_log": [rank0_only(on_log)],
        "on_eval_end": [rank0_only(on_eval_end)],
        "on_train_end": [rank0_only(on_close)],
        "on_exception": [rank0_only(on_close)],
    }


def is_bad_float(v: Any) -> bool:
    return isinstance(v, float) and (math.isnan(v) or math.isinf(v))
