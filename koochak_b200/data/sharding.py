"""Explicit, idempotent DDP input sharding (reference: koochak/data/sharding.py:18-119).

Item ``i`` of a dataset belongs to rank ``i % world_size``. Sharded wrappers
carry a marker attribute so sharding twice is a no-op and the loop can warn
about unsharded inputs under DDP.
"""

from __future__ import annotations

import warnings
from typing import Any, Iterable, Iterator

__all__ = ["is_sharded", "mark_sharded", "shard_iterable_dataset", "shard_map_dataset", "shard_dataset",
           "warn_if_unsharded", "ShardedIterable", "ShardedMapDataset"]

_MARK = "__koochak_sharded__"


def is_sharded(obj: Any) -> bool:
    if obj is None:
        return False
    if getattr(obj, _MARK, False):
        return True
    inner = getattr(obj, "dataset", None)
    return inner is not None and inner is not obj and is_sharded(inner)


def mark_sharded(obj: Any) -> Any:
    try:
        setattr(obj, _MARK, True)
    except (AttributeError, TypeError):
        pass  # builtins cannot carry attributes
    return obj


class ShardedIterable:
    def __init__(self, iterable: Iterable[Any], rank: int, world_size: int) -> None:
        self._src = iterable
        self._rank = int(rank)
        self._world = int(world_size)
        mark_sharded(self)

    def __iter__(self) -> Iterator[Any]:
        if self._world <= 1:
            yield from self._src
            return
        for i, item in enumerate(self._src):
            if i % self._world == self._rank:
                yield item


class ShardedMapDataset:
    def __init__(self, dataset: Any, rank: int, world_size: int) -> None:
        self._src = dataset
        self._rank = int(rank)
        self._world = int(world_size)
        mark_sharded(self)

    def __len__(self) -> int:
        n = len(self._src)
        return n if self._world <= 1 else max(0, (n - self._rank + self._world - 1) // self._world)

    def __getitem__(self, idx: int) -> Any:
        if self._world <= 1:
            return self._src[idx]
        j = idx * self._world + self._rank
        if j >= len(self._src):
            raise IndexError("sharded dataset index out of range")
        return self._src[j]


def shard_iterable_dataset(iterable: Iterable[Any], rank: int, world_size: int) -> Iterable[Any]:
    if is_sharded(iterable):
        return mark_sharded(iterable)
    if getattr(iterable, "dataset", None) is not None:
        warnings.warn("[koochak][ddp] sharding an outer DataLoader/iterable by batch. If the underlying dataset is "
                      "expensive, this can discard work and create rank skew.", stacklevel=2)
    return ShardedIterable(iterable, rank, world_size)


def shard_map_dataset(dataset: Any, rank: int, world_size: int) -> Any:
    if is_sharded(dataset):
        return mark_sharded(dataset)
    return ShardedMapDataset(dataset, rank, world_size)


def shard_dataset(dataset: Any, *, rank: int, world_size: int, mode: str) -> Any:
    if dataset is None:
        return None
    key = str(mode).lower()
    if key == "iterable":
        return shard_iterable_dataset(dataset, rank, world_size)
    if key == "map":
        return shard_map_dataset(dataset, rank, world_size)
    raise ValueError(f"Invalid shard_dataset mode: {mode!r} (expected 'iterable' or 'map')")


def warn_if_unsharded(dataset: Any, *, enabled: bool, name: str = "dataset") -> None:
    if enabled and dataset is not None and not is_sharded(dataset):
        warnings.warn(f"[koochak][ddp] {name} is not sharded; each rank may replay the full data. Enable "
                      "train.shard_dataset/train.shard_eval_dataset or shard explicitly via "
                      "koochak_b200.data.sharding.shard_dataset(...).", stacklevel=2)
