"""Environment flags and the opt-in ``compile_wrap`` decorator (reference: koochak/utils/flags.py:84-185).

``compile_wrap`` keeps the reference's API: a function decorated with it runs
eagerly unless ``KOOCHAK_USE_COMPILE=1``, in which case it is compiled once
with ``torch.compile`` and falls back to eager on compiler errors. The native
kernels of this package never depend on it.
"""

from __future__ import annotations

import os
import threading
import warnings
from contextlib import contextmanager
from functools import update_wrapper
from typing import Any, Callable

import torch

from ..core.precision import prepare_compile_backend

__all__ = ["compile_wrap", "get_use_compile", "get_compile_mode", "get_checkpointing", "get_compile_wrap_enabled",
           "set_compile_wrap_enabled", "in_checkpoint_recompute", "checkpoint_context_fn"]

_PREFIXES = ("KOOCHAK_", "SEE_MORE_ALPHA_", "KAVEH_")
_state = threading.local()
_WRAP_ENABLED = True


def _env(default: str, suffix: str) -> str:
    for prefix in _PREFIXES:
        v = os.environ.get(prefix + suffix)
        if v is not None:
            return v
    return default


def _fallback_types() -> tuple:
    types = []
    try:
        from torch._dynamo import exc as dyn

        types += [getattr(dyn, n, None) for n in ("BackendCompilerFailed", "InternalCompilerError", "ResetRequired")]
    except Exception:
        pass
    try:
        from torch._inductor import exc as ind

        types.append(getattr(ind, "InductorError", None))
    except Exception:
        pass
    return tuple(t for t in types if isinstance(t, type) and t is not RuntimeError)


_FALLBACK = _fallback_types()


def in_checkpoint_recompute() -> bool:
    return getattr(_state, "recompute", False)


@contextmanager
def _recompute_flag(value: bool):
    prev = in_checkpoint_recompute()
    _state.recompute = value
    try:
        yield
    finally:
        _state.recompute = prev


def checkpoint_context_fn():
    """Context pair for ``torch.utils.checkpoint``: (forward, recompute)."""

    return _recompute_flag(False), _recompute_flag(True)


def get_use_compile() -> bool:
    return _WRAP_ENABLED and _env("0", "USE_COMPILE") == "1"


def get_compile_mode() -> str:
    return _env("default", "COMPILE_MODE")


def get_checkpointing() -> bool:
    return _env("0", "USE_GRADIENT_CHECKPOINTING") == "1"


def get_compile_wrap_enabled() -> bool:
    return bool(_WRAP_ENABLED)


def set_compile_wrap_enabled(enabled: bool) -> None:
    global _WRAP_ENABLED
    _WRAP_ENABLED = bool(enabled)


class compile_wrap:
    """Descriptor/decorator: optional ``torch.compile`` with eager fallback."""

    def __init__(self, function: Callable[..., Any], *args, **kwargs) -> None:
        self.function = function
        self.args = args
        self.kwargs = kwargs
        self._compiled = None
        update_wrapper(self, function)

    def __get__(self, instance, owner):
        if instance is None:
            return self
        return self.function.__get__(instance, owner)

    @property
    def compiled_function(self):
        if self._compiled is None:
            self._compiled = self.function
            if get_use_compile():
                try:
                    kw = {"fullgraph": False, "dynamic": False, **self.kwargs}
                    kw.setdefault("mode", get_compile_mode())
                    prepare_compile_backend()
                    self._compiled = torch.compile(self.function, *self.args, **kw)
                except RuntimeError:
                    self._compiled = self.function
        return self._compiled

    def __call__(self, *args, **kwargs):
        fn = self.compiled_function
        if in_checkpoint_recompute() or (getattr(torch, "_dynamo", None) is not None and torch._dynamo.is_compiling()):
            return self.function(*args, **kwargs)
        if fn is self.function:
            return fn(*args, **kwargs)
        try:
            return fn(*args, **kwargs)
        except Exception as exc:
            if not self._should_fallback(exc):
                raise
            self._compiled = self.function
            if _env("0", "COMPILE_DEBUG") == "1":
                warnings.warn(f"Falling back to eager execution for {self.function.__qualname__}: {exc}",
                              RuntimeWarning)
            return self.function(*args, **kwargs)

    @staticmethod
    def _should_fallback(exc: Exception) -> bool:
        if _FALLBACK and isinstance(exc, _FALLBACK):
            return True
        return isinstance(exc, RuntimeError) and "No valid triton configs" in str(exc)
