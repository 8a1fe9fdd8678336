"""JSON-value validation and immutable views for job and artifact records.

(reference: koochak/jobs_types.py)

Imports nothing outside the standard library, so job submission code can use
it without PyTorch.
"""

from __future__ import annotations

import math
from types import MappingProxyType
from typing import Any, Mapping

__all__ = ["validate_json_value", "freeze_json", "thaw_json"]


def validate_json_value(value: Any, label: str = "value") -> None:
    """Raise ValueError unless ``value`` is plain JSON data (finite floats, string keys)."""

    stack = [(value, label)]
    while stack:
        v, where = stack.pop()
        if v is None or isinstance(v, (str, bool, int)):
            continue
        if type(v) is float:
            if not math.isfinite(v):
                raise ValueError(f"{where} must not contain NaN or infinity")
            continue
        if isinstance(v, Mapping):
            if not all(isinstance(k, str) for k in v):
                raise ValueError(f"{where} mappings must have string keys")
            stack.extend((item, f"{where}.{k}") for k, item in v.items())
            continue
        if isinstance(v, (list, tuple)):
            stack.extend((item, f"{where}[{i}]") for i, item in enumerate(v))
            continue
        raise ValueError(f"{where} contains a non-JSON value: {type(v).__name__}")


def _freeze(v: Any) -> Any:
    if isinstance(v, Mapping):
        return MappingProxyType({k: _freeze(x) for k, x in v.items()})
    if isinstance(v, (list, tuple)):
        return tuple(_freeze(x) for x in v)
    return v


def freeze_json(value: Any, label: str = "value") -> Any:
    """Validate, then return read-only mappings and tuples in place of dicts and lists."""

    validate_json_value(value, label)
    return _freeze(value)


def thaw_json(value: Any) -> Any:
    """Plain dicts and lists again, ready for ``json.dumps``."""

    if isinstance(value, Mapping):
        return {k: thaw_json(x) for k, x in value.items()}
    if isinstance(value, (list, tuple)):
        return [thaw_json(x) for x in value]
    return value
