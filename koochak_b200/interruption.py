"""Evacuation: a scheduler's SIGUSR1 becomes "checkpoint at the next update boundary, then exit 75".

(behaviour of reference koochak/interruption.py:22-178)

Three small parts:

* ``_Latch`` -- a flag that a signal handler may set (setting a bool is the
  only thing the handler does: anything more is not async-signal-safe) and
  that code may set directly;
* ``_RunnerFiles`` -- the directory shared with the managed runner
  (``$KOOCHAK_EVACUATION_DIR``): the runner drops ``requested`` when it wants
  the job out, the job drops ``evacuated`` once its checkpoint is safe;
* ``agree_any`` -- every rank learns whether any rank raised any of a few
  flags, with one MAX all-reduce of an int64 vector (on the GPU under NCCL).

``EvacuationController.reconcile_requests`` is what the training loop calls
after each update: it reads the runner's file, agrees on ``[evacuate,
*extra]`` across ranks, and keeps a positive answer latched so a signal that
arrived after the local read still counts at the next boundary.

Exit codes 75 (evacuated), 76 (checkpoint acknowledgement timeout) and 77
(restart after an out-of-memory error) are contracts with schedulers.
"""

from __future__ import annotations

import os
import signal
import threading
from pathlib import Path
from typing import Optional, Sequence, Tuple, Union

__all__ = [
    "CHECKPOINT_ACK_TIMEOUT_EXIT_CODE", "EVACUATION_EXIT_CODE", "EVACUATION_DIR_ENV", "EVACUATED_FILE",
    "EVACUATION_REQUEST_FILE", "EvacuationController", "OOM_RESTART_EXIT_CODE", "install_evacuation_handler",
    "agree_any",
]

EVACUATION_EXIT_CODE = 75
CHECKPOINT_ACK_TIMEOUT_EXIT_CODE = 76
OOM_RESTART_EXIT_CODE = 77
EVACUATION_DIR_ENV = "KOOCHAK_EVACUATION_DIR"
EVACUATION_REQUEST_FILE = "requested"
EVACUATED_FILE = "evacuated"


def _signal_number(name: Union[str, int]) -> int:
    """SIGUSR1 from ``"USR1"``, ``"SIGUSR1"`` or the number; any other signal is refused."""

    if isinstance(name, int):
        number: object = name
    else:
        text = str(name).upper()
        number = getattr(signal, text if text.startswith("SIG") else f"SIG{text}", None)
        if not isinstance(number, int):
            raise ValueError(f"unsupported evacuation signal: {name!r}")
    if number != signal.SIGUSR1:
        raise ValueError("evacuation signal must be SIGUSR1")
    return int(number)


class _Latch:
    """A settable flag with an optional signal handler that only sets it."""

    def __init__(self, signum: int) -> None:
        self.signum = signum
        self.value = False
        self._saved: object = signal.SIG_DFL
        self.armed = False

    def _handler(self, _signum: int, _frame: object) -> None:
        self.value = True

    def arm(self) -> None:
        if threading.current_thread() is not threading.main_thread():
            raise RuntimeError("evacuation signal handler must be installed from the main thread")
        self._saved = signal.getsignal(self.signum)
        signal.signal(self.signum, self._handler)
        self.armed = True

    def disarm(self) -> None:
        if self.armed and threading.current_thread() is threading.main_thread():
            signal.signal(self.signum, self._saved)
        self.armed = False


class _RunnerFiles:
    """The control directory shared with the managed runner (absent outside it)."""

    def __init__(self, directory: Optional[str]) -> None:
        self.root = Path(directory) if directory else None

    def _has(self, name: str) -> bool:
        return self.root is not None and (self.root / name).exists()

    def stop_requested(self) -> bool:
        return self._has(EVACUATION_REQUEST_FILE)

    def evacuated(self) -> bool:
        return self._has(EVACUATED_FILE)

    def announce_evacuated(self) -> None:
        if self.root is not None:
            (self.root / EVACUATED_FILE).touch()


def agree_any(flags: Sequence[bool]) -> Tuple[bool, ...]:
    """Element-wise OR of ``flags`` over all ranks (the flags themselves without a process group)."""

    from .core import dist as dist_lib

    local = tuple(bool(f) for f in flags)
    if not (dist_lib.is_initialized() and dist_lib.world_size() > 1):
        return local
    import torch

    on_gpu = str(torch.distributed.get_backend()).lower() == "nccl"
    vec = torch.tensor(local, dtype=torch.int64, device="cuda" if on_gpu else "cpu")
    torch.distributed.all_reduce(vec, op=torch.distributed.ReduceOp.MAX)
    return tuple(bool(v) for v in vec.tolist())


class EvacuationController:
    """Opt-in SIGUSR1 latch plus the per-update cross-rank agreement on stopping."""

    def __init__(self, enabled: bool = False, *, signal_name: Union[str, int] = "USR1",
                 exit_code: int = EVACUATION_EXIT_CODE) -> None:
        if int(exit_code) != EVACUATION_EXIT_CODE:
            raise ValueError(f"evacuation exit code is reserved: {EVACUATION_EXIT_CODE}")
        self.enabled = bool(enabled)
        self.exit_code = EVACUATION_EXIT_CODE
        self._latch = _Latch(_signal_number(signal_name))
        self._files = _RunnerFiles(None)

    @property
    def signal_number(self) -> int:
        return self._latch.signum

    @property
    def requested(self) -> bool:
        return self._latch.value

    def request(self) -> None:
        self._latch.value = True

    def install(self) -> "EvacuationController":
        if self.enabled and not self._latch.armed:
            self._latch.arm()
            self._files = _RunnerFiles(os.environ.get(EVACUATION_DIR_ENV))
        return self

    def uninstall(self) -> None:
        if self._latch.armed:
            self._files = _RunnerFiles(None)
            self._latch.disarm()

    @property
    def already_evacuated(self) -> bool:
        return self._files.evacuated()

    def mark_evacuated(self) -> None:
        self._files.announce_evacuated()

    def reconcile(self) -> bool:
        return self.reconcile_requests()[0]

    def reconcile_requests(self, *requests: bool) -> Tuple[bool, ...]:
        """Agree across ranks on ``[evacuate, *requests]``; an agreed evacuation stays latched."""

        if self._files.stop_requested():
            self._latch.value = True
        agreed = agree_any((self._latch.value, *requests))
        self._latch.value = self._latch.value or agreed[0]
        return agreed


def install_evacuation_handler(enabled: bool = True, *, signal_name: Union[str, int] = "USR1") -> EvacuationController:
    return EvacuationController(enabled, signal_name=signal_name).install()
