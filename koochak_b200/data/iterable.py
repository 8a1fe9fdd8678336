"""Host-to-device batch transfer and CUDA prefetching.

(behaviour of reference koochak/data/iterable.py:17-295)

``CudaPrefetcher`` keeps up to ``prefetch`` batches in flight. Staging a
batch means: copy its tensors to the device on a side stream (non-blocking,
so pinned host memory overlaps with compute), optionally run
``prepare_fn`` on that stream, and record an event. The consumer's stream
waits on that event before the batch is handed over, and every tensor is
recorded on the consumer stream so the allocator does not reuse it early.

Where the work runs (``threaded`` / ``pipeline``):

* inline -- staging happens in ``__next__`` on the training thread;
* ``single`` -- one worker thread fetches and stages;
* ``two_stage`` -- a fetch thread (``next(iterator)``, CPU work) feeds a
  staging thread (the CUDA submission) through a second bounded queue.

Every thread stops at ``close``; an exception in a worker is re-raised on the
consumer's thread. Dict batches receive ``koochak_prefetch_*`` diagnostics
(wait time, queue depths, batch age, staging cost).
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass
from queue import Empty, Full, Queue
from threading import Event, Thread
from typing import Any, Callable, Iterable, Iterator, List, Optional

import torch

__all__ = ["to_device", "prefetch", "cycle", "take", "CudaPrefetcher"]

BatchPrepareFn = Callable[[Any], Any]
_DONE = object()  # end-of-stream marker passed through the queues


def _map_tensors(batch: Any, fn: Callable[[torch.Tensor], Any]) -> Any:
    if isinstance(batch, torch.Tensor):
        return fn(batch)
    if isinstance(batch, dict):
        return {k: _map_tensors(v, fn) for k, v in batch.items()}
    if isinstance(batch, (list, tuple)):
        mapped = [_map_tensors(v, fn) for v in batch]
        return tuple(mapped) if isinstance(batch, tuple) else mapped
    return batch


def to_device(batch: Any, device: torch.device) -> Any:
    """Move every tensor inside nested dicts / lists / tuples to ``device`` (non-blocking)."""

    return _map_tensors(batch, lambda t: t.to(device, non_blocking=True))


@dataclass
class _Ready:
    batch: Any
    event: "torch.cuda.Event"
    staged_at: float
    staging_cost_s: float
    fetch_backlog: int = -1


class _Channel:
    """A bounded queue whose blocking calls give up once ``stop`` is set."""

    def __init__(self, capacity: int, stop: Event) -> None:
        self.q: Queue = Queue(maxsize=capacity)
        self.stop = stop

    def put(self, item: Any) -> bool:
        while not self.stop.is_set():
            try:
                self.q.put(item, timeout=0.1)
                return True
            except Full:
                continue
        return False

    def get(self) -> Any:
        while not self.stop.is_set():
            try:
                return self.q.get(timeout=0.1)
            except Empty:
                continue
        return _DONE

    def size(self) -> int:
        return self.q.qsize()


class CudaPrefetcher:
    def __init__(self, iterator: Iterator[Any], device: torch.device, prefetch: int = 2, *,
                 prepare_fn: Optional[BatchPrepareFn] = None, threaded: bool = False, pipeline: str = "single"):
        self.iterator = iterator
        self.device = device
        self.prefetch = max(1, int(prefetch))
        self.prepare_fn = prepare_fn
        self.threaded = bool(threaded)
        self.pipeline = str(pipeline or "single").strip().lower().replace("-", "_")
        self.stream = torch.cuda.Stream(device=device)
        self._stop = Event()
        self._error: Optional[BaseException] = None
        self._threads: List[Thread] = []
        self._closed = False
        if not self.threaded:
            self._pending: deque = deque()
            self._source_done = False
            self._refill()
            return
        self._out = _Channel(self.prefetch, self._stop)
        if self.pipeline in ("two_stage", "staged"):
            self._fetched = _Channel(self.prefetch, self._stop)
            self._spawn(self._fetch_loop, self._fetched)
            self._spawn(self._stage_loop, self._out)
        else:
            self._fetched = None
            self._spawn(self._fetch_and_stage_loop, self._out)

    # ---------------------------------------------------------------- staging
    def _stage(self, batch: Any) -> _Ready:
        began = time.perf_counter()
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            batch = to_device(batch, self.device)
            if self.prepare_fn is not None:
                prepared = self.prepare_fn(batch)
                batch = batch if prepared is None else prepared
            landed = torch.cuda.Event()
            landed.record(self.stream)
        now = time.perf_counter()
        return _Ready(batch, landed, now, now - began)

    # ---------------------------------------------------------------- inline mode
    def _refill(self) -> None:
        while len(self._pending) < self.prefetch and not self._source_done:
            try:
                self._pending.append(self._stage(next(self.iterator)))
            except StopIteration:
                self._source_done = True

    # ---------------------------------------------------------------- threaded modes
    def _spawn(self, body: Callable[[], None], feeds: _Channel) -> None:
        t = Thread(target=self._guarded, args=(body, feeds), daemon=True)
        self._threads.append(t)
        t.start()

    def _guarded(self, body: Callable[[], None], feeds: _Channel) -> None:
        try:
            body()
        except BaseException as exc:  # re-raised on the consumer's thread, after the batches before it
            if self._error is None:
                self._error = exc
            feeds.put(_DONE)

    def _fetch_and_stage_loop(self) -> None:
        for batch in self.iterator:
            if not self._out.put(self._stage(batch)):
                return
        self._out.put(_DONE)

    def _fetch_loop(self) -> None:
        assert self._fetched is not None
        while not self._stop.is_set():
            began = time.perf_counter()
            try:
                batch = next(self.iterator)
            except StopIteration:
                self._fetched.put(_DONE)
                return
            if isinstance(batch, dict):
                batch["koochak_prefetch_cpu_fetch_time_s"] = float(time.perf_counter() - began)
            if not self._fetched.put(batch):
                return

    def _stage_loop(self) -> None:
        assert self._fetched is not None
        while not self._stop.is_set():
            batch = self._fetched.get()
            if batch is _DONE:
                self._out.put(_DONE)
                return
            ready = self._stage(batch)
            ready.fetch_backlog = self._fetched.size()
            if not self._out.put(ready):
                return

    # ---------------------------------------------------------------- consumer
    def __iter__(self) -> "CudaPrefetcher":
        return self

    def __next__(self) -> Any:
        if not self.threaded:
            if not self._pending:
                raise StopIteration
            ready = self._pending.popleft()
            batch = self._deliver(ready, 0.0, len(self._pending))
            self._refill()
            return batch
        began = time.perf_counter()
        ready = self._out.get()
        waited = time.perf_counter() - began
        if ready is _DONE:
            if self._error is not None:
                raise self._error
            raise StopIteration
        return self._deliver(ready, waited, self._out.size())

    def _deliver(self, ready: _Ready, waited: float, depth: int) -> Any:
        consumer = torch.cuda.current_stream(self.device)
        if isinstance(ready.batch, dict):
            ready.batch.update({
                "koochak_prefetch_get_wait_s": float(waited),
                "koochak_prefetch_event_ready": float(bool(ready.event.query())),
                "koochak_prefetch_queue_depth": float(depth),
                "koochak_prefetch_cpu_queue_depth": float(ready.fetch_backlog),
                "koochak_prefetch_age_s": float(max(0.0, time.perf_counter() - ready.staged_at)),
                "koochak_prefetch_prepare_submit_s": float(ready.staging_cost_s),
            })
        consumer.wait_event(ready.event)
        _map_tensors(ready.batch, lambda t: t.record_stream(consumer))
        return ready.batch

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            self._stop.set()
            for t in self._threads:
                t.join(timeout=5.0)


def prefetch(iterable: Iterator[Any], device: torch.device, prefetch: int = 2, *,
             prepare_fn: Optional[BatchPrepareFn] = None, threaded: bool = False,
             pipeline: str = "single") -> Iterator[Any]:
    """A ``CudaPrefetcher`` over ``iterable`` on CUDA devices (the iterable itself otherwise)."""

    if getattr(device, "type", "cpu") != "cuda" or prefetch <= 0:
        return iterable
    return CudaPrefetcher(iterable, device=device, prefetch=prefetch, prepare_fn=prepare_fn, threaded=threaded,
                          pipeline=pipeline)


def cycle(iterable: Iterable[Any]) -> Iterator[Any]:
    while True:
        yield from iterable


def take(iterable: Iterable[Any], n: int) -> Iterator[Any]:
    it = iter(iterable)
    for _ in range(max(0, n)):
        try:
            yield next(it)
        except StopIteration:
            return
