"""Compatibility location of the config helpers (reference: koochak/utils/config.py)."""

from __future__ import annotations

from .. import config as _config

get = _config.get
as_dict = _config.as_dict

__all__ = ["get", "as_dict"]
