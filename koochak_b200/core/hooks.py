"""Event hooks: ``{event: [callables]}`` dictionaries (reference: koochak/core/hooks.py:10-61).

``emit`` swallows callback exceptions unless ``suppress_exceptions=False`` or
the callback carries ``_koochak_fail_closed = True``.
"""

from __future__ import annotations

from typing import Callable, Dict, List, Optional

Hooks = Dict[str, List[Callable]]

__all__ = ["merge", "emit", "add", "rank0_only", "fail_closed"]


def merge(a: Optional[Hooks], b: Optional[Hooks]) -> Hooks:
    """Concatenate two hook dicts; callbacks of ``a`` run first."""

    out: Hooks = {}
    for src in (a, b):
        for event, fns in (src or {}).items():
            out.setdefault(event, []).extend(fns)
    return out


def add(hooks: Hooks, event: str, fn: Callable) -> Hooks:
    hooks.setdefault(event, []).append(fn)
    return hooks


def emit(hooks: Optional[Hooks], event: str, *args, suppress_exceptions: bool = True, **kwargs) -> None:
    if not hooks:
        return
    for fn in list(hooks.get(event) or ()):
        try:
            fn(*args, **kwargs)
        except Exception:
            if not suppress_exceptions or getattr(fn, "_koochak_fail_closed", False):
                raise


def rank0_only(fn: Callable) -> Callable:
    from . import dist as dist_lib

    def _wrapped(*args, **kwargs):
        if dist_lib.rank0():
            return fn(*args, **kwargs)
        return None

    return _wrapped


def fail_closed(fn: Callable) -> Callable:
    """Mark a callback so that its exceptions propagate out of ``emit``."""

    fn._koochak_fail_closed = True  # type: ignore[attr-defined]
    return fn
