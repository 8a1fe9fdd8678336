"""Human-written byte sizes: ``4096``, ``64M``, ``512MiB``, ``1.5GB``.

Single-letter and ``*iB`` units are binary, ``KB/MB/GB/TB`` are decimal
(reference: koochak/utils/sizes.py:13-49).
"""

from __future__ import annotations

import math
import re
from typing import Union

__all__ = ["parse_size"]

_BINARY = {"K": 1, "KIB": 1, "M": 2, "MIB": 2, "G": 3, "GIB": 3, "T": 4, "TIB": 4}
_DECIMAL = {"KB": 1, "MB": 2, "GB": 3, "TB": 4}
_PATTERN = re.compile(r"^\s*(\d+(?:\.\d+)?)\s*([A-Za-z]*)\s*$")


def _multiplier(unit: str) -> int:
    u = unit.upper()
    if u in ("", "B"):
        return 1
    if u in _BINARY:
        return 1024 ** _BINARY[u]
    if u in _DECIMAL:
        return 1000 ** _DECIMAL[u]
    raise KeyError(u)


def parse_size(value: Union[str, int]) -> int:
    """Return a non-negative byte count."""

    if isinstance(value, bool):
        raise ValueError(f"invalid size: {value!r}")
    if isinstance(value, int):
        if value < 0:
            raise ValueError(f"size must be non-negative: {value!r}")
        return value
    if not isinstance(value, str):
        raise ValueError(f"size must be an integer or a string, got {type(value).__name__}")
    m = _PATTERN.match(value)
    try:
        if m is None:
            raise KeyError(value)
        size = float(m.group(1)) * _multiplier(m.group(2))
    except KeyError:
        raise ValueError(f"invalid size {value!r}; use e.g. 4096, 64M, 512MiB, or 1.5GB") from None
    if not math.isfinite(size):
        raise ValueError(f"invalid size: {value!r}")
    return int(size)
