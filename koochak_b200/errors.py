"""Exceptions raised by the native layer."""

from __future__ import annotations

_CODES = {
    1: "TMA producer timed out waiting for a free pipeline stage",
    2: "MMA issuer timed out waiting for operands or an accumulator",
    3: "epilogue timed out waiting for an accumulator",
    4: "kernel drain at exit did not complete",
    5: "cross-GPU wait ran out (a peer did not arrive)",
    6: "kernel rejected its arguments (index out of range)",
    7: "debug-bounds build: an index fell outside its declared extent",
    8: "row-streaming kernel timed out waiting for a staged row",
}


class KernelTimeoutError(RuntimeError):
    """A native kernel gave up a bounded wait and returned an error status."""

    def __init__(self, code: int) -> None:
        self.code = int(code)
        super().__init__(f"koochak_b200 kernel status {self.code}: {_CODES.get(self.code, 'unknown error')}")


class CommTimeoutError(KernelTimeoutError):
    """A cross-GPU flag wait inside a communication kernel ran out."""
