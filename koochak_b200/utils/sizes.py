"""Byte sizes written by people: ``4096``, ``64M``, ``512MiB``, ``1.5GB``.

(behaviour of reference koochak/utils/sizes.py:13-49: bare letters and
``*iB`` are powers of 1024, ``KB/MB/GB/TB`` powers of 1000)

The text is split into a decimal number and a unit suffix by hand; the
suffix is looked up in one table of multipliers.
"""

from __future__ import annotations

import math
from typing import Union

__all__ = ["parse_size"]


def _unit_table() -> dict:
    table = {"": 1, "B": 1}
    for power, letter in enumerate("KMGT", start=1):
        table[letter] = table[letter + "IB"] = 1024 ** power
        table[letter + "B"] = 1000 ** power
    return table


_UNITS = _unit_table()
_HINT = "use e.g. 4096, 64M, 512MiB, or 1.5GB"


def _split(text: str):
    """('1.5', 'GB') from ' 1.5 GB '; None when the text is not number + letters."""

    body = text.strip()
    cut = len(body)
    while cut > 0 and body[cut - 1].isalpha():
        cut -= 1
    number, unit = body[:cut].rstrip(), body[cut:]
    if not number or number.count(".") > 1 or not number.replace(".", "").isdigit():
        return None
    if number.startswith(".") or number.endswith("."):
        return None
    return number, unit.upper()


def parse_size(value: Union[str, int]) -> int:
    """Byte count of ``value`` (an int, or a number with an optional unit); never negative."""

    if isinstance(value, bool) or not isinstance(value, (int, str)):
        kind = type(value).__name__
        raise ValueError(f"invalid size: {value!r}" if isinstance(value, bool)
                         else f"size must be an integer or a string, got {kind}")
    if isinstance(value, int):
        if value < 0:
            raise ValueError(f"size must be non-negative: {value!r}")
        return value
    parts = _split(value)
    if parts is None or parts[1] not in _UNITS:
        raise ValueError(f"invalid size {value!r}; {_HINT}")
    amount = float(parts[0]) * _UNITS[parts[1]]
    if not math.isfinite(amount):
        raise ValueError(f"invalid size: {value!r}")
    return int(amount)
