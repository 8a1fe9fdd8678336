"""Data helpers: device transfer and prefetch, sharding, shard files, packed collections."""

from .iterable import cycle, prefetch, take, to_device  # noqa: F401
from .sharding import shard_dataset  # noqa: F401
