"""Explicit, idempotent input sharding for data parallelism.

(behaviour of reference koochak/data/sharding.py:18-119)

Rank ``r`` of ``W`` sees items ``r, r + W, r + 2W, ...`` of a dataset. A
sharded wrapper carries a marker attribute, so sharding an already sharded
dataset is a no-op and the training loop can warn when data-parallel ranks
would all replay the full data.
"""

from __future__ import annotations

import itertools
import warnings
from typing import Any, Iterable, Iterator

__all__ = ["is_sharded", "mark_sharded", "shard_iterable_dataset", "shard_map_dataset", "shard_dataset",
           "warn_if_unsharded", "ShardedIterable", "ShardedMapDataset"]

_SHARDED = "__koochak_sharded__"


def is_sharded(obj: Any) -> bool:
    """True for a sharded wrapper, or an object (e.g. a DataLoader) whose ``.dataset`` chain leads to one."""

    seen = set()
    while obj is not None and id(obj) not in seen:
        if getattr(obj, _SHARDED, False):
            return True
        seen.add(id(obj))
        obj = getattr(obj, "dataset", None)
    return False


def mark_sharded(obj: Any) -> Any:
    try:
        setattr(obj, _SHARDED, True)
    except (AttributeError, TypeError):
        pass  # objects without a __dict__ cannot carry the marker
    return obj


class _Shard:
    def __init__(self, source: Any, rank: int, world_size: int) -> None:
        self._src, self._rank, self._world = source, int(rank), int(world_size)
        mark_sharded(self)

    @property
    def _whole(self) -> bool:
        return self._world <= 1


class ShardedIterable(_Shard):
    """Every ``world_size``-th item of an iterable, starting at ``rank``."""

    def __iter__(self) -> Iterator[Any]:
        source = iter(self._src)
        return source if self._whole else itertools.islice(source, self._rank, None, self._world)


class ShardedMapDataset(_Shard):
    """Index ``i`` maps to item ``i * world_size + rank`` of the source."""

    def __len__(self) -> int:
        total = len(self._src)
        return total if self._whole else max(0, -(-(total - self._rank) // self._world))

    def __getitem__(self, idx: int) -> Any:
        if self._whole:
            return self._src[idx]
        source_index = idx * self._world + self._rank
        if source_index >= len(self._src):
            raise IndexError("sharded dataset index out of range")
        return self._src[source_index]


def shard_iterable_dataset(iterable: Iterable[Any], rank: int, world_size: int) -> Iterable[Any]:
    if is_sharded(iterable):
        return mark_sharded(iterable)
    if getattr(iterable, "dataset", None) is not None:
        warnings.warn("[koochak][ddp] sharding an outer DataLoader/iterable by batch. If the underlying dataset is "
                      "expensive, this can discard work and create rank skew.", stacklevel=2)
    return ShardedIterable(iterable, rank, world_size)


def shard_map_dataset(dataset: Any, rank: int, world_size: int) -> Any:
    return mark_sharded(dataset) if is_sharded(dataset) else ShardedMapDataset(dataset, rank, world_size)


_BY_MODE = {"iterable": shard_iterable_dataset, "map": shard_map_dataset}


def shard_dataset(dataset: Any, *, rank: int, world_size: int, mode: str) -> Any:
    if dataset is None:
        return None
    make = _BY_MODE.get(str(mode).lower())
    if make is None:
        raise ValueError(f"Invalid shard_dataset mode: {mode!r} (expected 'iterable' or 'map')")
    return make(dataset, rank, world_size)


def warn_if_unsharded(dataset: Any, *, enabled: bool, name: str = "dataset") -> None:
    if enabled and dataset is not None and not is_sharded(dataset):
        warnings.warn(f"[koochak][ddp] {name} is not sharded; each rank may replay the full data. Enable "
                      "train.shard_dataset/train.shard_eval_dataset or shard explicitly via "
                      "koochak_b200.data.sharding.shard_dataset(...).", stacklevel=2)
