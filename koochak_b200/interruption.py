"""Evacuation signalling: SIGUSR1 -> checkpoint at the next safe boundary -> exit 75.

(reference: koochak/interruption.py:22-178)

The signal handler only sets a flag. ``reconcile_requests`` is called by the
loop after every update: it folds in a request file from the managed runner
(``$KOOCHAK_EVACUATION_DIR/requested``) and agrees on the flags across ranks
with one MAX all-reduce of a small int64 vector. A request that arrives after
the local flag was read is kept for the next reduction.
"""

from __future__ import annotations

import os
import signal
import threading
from pathlib import Path

__all__ = [
    "CHECKPOINT_ACK_TIMEOUT_EXIT_CODE", "EVACUATION_EXIT_CODE", "EVACUATION_DIR_ENV", "EVACUATED_FILE",
    "EVACUATION_REQUEST_FILE", "EvacuationController", "OOM_RESTART_EXIT_CODE", "install_evacuation_handler",
]

EVACUATION_EXIT_CODE = 75
CHECKPOINT_ACK_TIMEOUT_EXIT_CODE = 76
OOM_RESTART_EXIT_CODE = 77
EVACUATION_DIR_ENV = "KOOCHAK_EVACUATION_DIR"
EVACUATION_REQUEST_FILE = "requested"
EVACUATED_FILE = "evacuated"


def _resolve_signal(name: str | int) -> int:
    if isinstance(name, int):
        num = name
    else:
        text = str(name).upper()
        text = text if text.startswith("SIG") else "SIG" + text
        num = getattr(signal, text, None)
        if not isinstance(num, int):
            raise ValueError(f"unsupported evacuation signal: {name!r}")
    if num != signal.SIGUSR1:
        raise ValueError("evacuation signal must be SIGUSR1")
    return int(num)


class EvacuationController:
    """Opt-in SIGUSR1 handler plus the cross-rank stop-flag reduction."""

    def __init__(self, enabled: bool = False, *, signal_name: str | int = "USR1",
                 exit_code: int = EVACUATION_EXIT_CODE) -> None:
        self.enabled = bool(enabled)
        self.signal_number = _resolve_signal(signal_name)
        if int(exit_code) != EVACUATION_EXIT_CODE:
            raise ValueError(f"evacuation exit code is reserved: {EVACUATION_EXIT_CODE}")
        self.exit_code = EVACUATION_EXIT_CODE
        self._requested = False
        self._previous_handler: object = signal.SIG_DFL
        self._installed = False
        self._control_dir: Path | None = None

    @property
    def requested(self) -> bool:
        return self._requested

    def request(self) -> None:
        self._requested = True

    def _on_signal(self, _signum: int, _frame: object) -> None:
        self._requested = True  # nothing else is async-signal-safe

    def install(self) -> "EvacuationController":
        if not self.enabled or self._installed:
            return self
        if threading.current_thread() is not threading.main_thread():
            raise RuntimeError("evacuation signal handler must be installed from the main thread")
        self._previous_handler = signal.getsignal(self.signal_number)
        signal.signal(self.signal_number, self._on_signal)
        self._installed = True
        directory = os.environ.get(EVACUATION_DIR_ENV)
        if directory:
            self._control_dir = Path(directory)
        return self

    @property
    def already_evacuated(self) -> bool:
        return self._control_dir is not None and (self._control_dir / EVACUATED_FILE).exists()

    def mark_evacuated(self) -> None:
        if self._control_dir is not None:
            (self._control_dir / EVACUATED_FILE).touch()

    def uninstall(self) -> None:
        if not self._installed:
            return
        self._control_dir = None
        if threading.current_thread() is threading.main_thread():
            signal.signal(self.signal_number, self._previous_handler)
        self._installed = False

    def reconcile(self) -> bool:
        return self.reconcile_requests()[0]

    def reconcile_requests(self, *requests: bool) -> tuple[bool, ...]:
        """MAX-reduce ``[evacuate, *requests]`` over ranks; returns the agreed flags."""

        import torch

        from .core import dist as dist_lib

        if (not self._requested and self._control_dir is not None
                and (self._control_dir / EVACUATION_REQUEST_FILE).exists()):
            self._requested = True
        flags = [bool(self._requested), *(bool(r) for r in requests)]
        if dist_lib.is_initialized() and dist_lib.world_size() > 1:
            backend = str(torch.distributed.get_backend()).lower()
            dev = "cuda" if backend == "nccl" else "cpu"
            t = torch.tensor([int(f) for f in flags], dtype=torch.int64, device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            flags = [bool(x) for x in t.tolist()]
        if flags[0]:
            self._requested = True
        return tuple(flags)


def install_evacuation_handler(enabled: bool = True, *, signal_name: str | int = "USR1") -> EvacuationController:
    return EvacuationController(enabled, signal_name=signal_name).install()
