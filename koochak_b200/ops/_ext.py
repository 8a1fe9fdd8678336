"""Access to the native sm_100a library, failing loudly when it is missing.

CUDA tensors always run through the native kernels; there is no silent
fallback to PyTorch on a GPU. CPU tensors use the PyTorch reference
implementations next to each op (they are also the numerical oracles of the
tests).
"""

from __future__ import annotations

import threading
from types import ModuleType
from typing import Optional

import torch

_lock = threading.Lock()
_mod: Optional[ModuleType] = None


def native() -> ModuleType:
    """Return the loaded ``koochak_b200_C`` module or raise ImportError."""

    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is None:
            from .. import _native_build

            _mod = _native_build.load()
    return _mod


def available() -> bool:
    try:
        native()
        return True
    except ImportError:
        return False


def check_status(device: Optional[torch.device] = None) -> None:
    """Raise if a kernel on ``device`` recorded a bounded-wait timeout."""

    if not torch.cuda.is_available():
        return
    idx = torch.cuda.current_device() if device is None or device.index is None else device.index
    code = native().read_and_clear_status(idx)
    if code:
        from ..errors import KernelTimeoutError

        raise KernelTimeoutError(code)


def use_native(t: torch.Tensor) -> bool:
    """Native kernels run for CUDA tensors; CPU tensors use the reference path."""

    return t.is_cuda
