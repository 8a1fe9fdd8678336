"""Host-to-device batch transfer and CUDA prefetching (reference: koochak/data/iterable.py:17-295).

``CudaPrefetcher`` copies upcoming batches on a side stream (and optionally
runs ``prepare_fn`` there), records an event per batch, and hands each batch
to the consumer after making the consumer's stream wait on that event.
Modes: inline (``threaded=False``), one worker thread (``pipeline="single"``),
or a CPU fetch thread feeding a CUDA submit thread (``"two_stage"``). Dict
batches receive ``koochak_prefetch_*`` timing diagnostics.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass
from queue import Empty, Full, Queue
from threading import Event, Lock, Thread
from typing import Any, Callable, Iterable, Iterator, Optional

import torch

__all__ = ["to_device", "prefetch", "cycle", "take", "CudaPrefetcher"]

BatchPrepareFn = Callable[[Any], Any]
_END = object()


def to_device(batch: Any, device: torch.device) -> Any:
    """Recursively move tensors in dicts/lists/tuples (non-blocking)."""

    if isinstance(batch, torch.Tensor):
        return batch.to(device, non_blocking=True)
    if isinstance(batch, dict):
        return {k: to_device(v, device) for k, v in batch.items()}
    if isinstance(batch, (list, tuple)):
        moved = [to_device(v, device) for v in batch]
        return tuple(moved) if isinstance(batch, tuple) else moved
    return batch


def _record_stream(batch: Any, stream: "torch.cuda.Stream") -> None:
    if isinstance(batch, torch.Tensor):
        batch.record_stream(stream)
    elif isinstance(batch, dict):
        for v in batch.values():
            _record_stream(v, stream)
    elif isinstance(batch, (list, tuple)):
        for v in batch:
            _record_stream(v, stream)


@dataclass
class _Staged:
    batch: Any
    event: "torch.cuda.Event"
    submitted_at: float
    submit_cost_s: float
    cpu_queue_depth: int = -1


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
        self._err_lock = Lock()
        self._stop = Event()
        self._error: Optional[BaseException] = None
        self._exhausted = False
        self._closed = False
        self.cpu_queue: Optional[Queue] = None
        if self.threaded:
            self.queue: Any = Queue(maxsize=self.prefetch)
            if self.pipeline in ("two_stage", "staged"):
                self.cpu_queue = Queue(maxsize=self.prefetch)
                self._cpu_worker = Thread(target=self._cpu_loop, daemon=True)
                self._cuda_worker = Thread(target=self._cuda_loop, daemon=True)
                self._cpu_worker.start()
                self._cuda_worker.start()
            else:
                self._worker = Thread(target=self._single_loop, daemon=True)
                self._worker.start()
        else:
            self.queue = deque()
            while len(self.queue) < self.prefetch and not self._exhausted:
                self._stage_next()

    # -- staging -----------------------------------------------------------
    def _stage(self, batch: Any) -> _Staged:
        t0 = time.perf_counter()
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            batch = to_device(batch, self.device)
            if self.prepare_fn is not None:
                out = self.prepare_fn(batch)
                if out is not None:
                    batch = out
            ev = torch.cuda.Event()
            ev.record(self.stream)
        t1 = time.perf_counter()
        return _Staged(batch, ev, t1, t1 - t0)

    def _stage_next(self) -> None:
        if self._exhausted:
            return
        try:
            batch = next(self.iterator)
        except StopIteration:
            self._exhausted = True
            return
        self.queue.append(self._stage(batch))

    # -- worker threads ----------------------------------------------------
    def _fail(self, exc: BaseException) -> None:
        with self._err_lock:
            if self._error is None:
                self._error = exc

    def _put(self, q: Queue, item: Any) -> bool:
        while not self._stop.is_set():
            try:
                q.put(item, timeout=0.1)
                return True
            except Full:
                pass
        return False

    def _get(self, q: Queue) -> Any:
        while not self._stop.is_set():
            try:
                return q.get(timeout=0.1)
            except Empty:
                pass
        return _END

    def _single_loop(self) -> None:
        try:
            while not self._stop.is_set():
                try:
                    batch = next(self.iterator)
                except StopIteration:
                    self._put(self.queue, _END)
                    return
                if not self._put(self.queue, self._stage(batch)):
                    return
        except BaseException as exc:  # surfaced on the consumer thread
            self._fail(exc)
            self._put(self.queue, _END)

    def _cpu_loop(self) -> None:
        assert self.cpu_queue is not None
        try:
            while not self._stop.is_set():
                t0 = time.perf_counter()
                try:
                    batch = next(self.iterator)
                except StopIteration:
                    self._put(self.cpu_queue, _END)
                    return
                if isinstance(batch, dict):
                    batch["koochak_prefetch_cpu_fetch_time_s"] = float(time.perf_counter() - t0)
                if not self._put(self.cpu_queue, batch):
                    return
        except BaseException as exc:
            self._fail(exc)
            self._put(self.cpu_queue, _END)

    def _cuda_loop(self) -> None:
        assert self.cpu_queue is not None
        try:
            while not self._stop.is_set():
                batch = self._get(self.cpu_queue)
                if batch is _END:
                    self._put(self.queue, _END)
                    return
                staged = self._stage(batch)
                staged.cpu_queue_depth = self.cpu_queue.qsize()
                if not self._put(self.queue, staged):
                    return
        except BaseException as exc:
            self._fail(exc)
            self._put(self.queue, _END)

    # -- consumer ----------------------------------------------------------
    def __iter__(self) -> "CudaPrefetcher":
        return self

    def __next__(self) -> Any:
        if self.threaded:
            t0 = time.perf_counter()
            item = self._get(self.queue)
            waited = time.perf_counter() - t0
            if item is _END:
                if self._error is not None:
                    raise self._error
                raise StopIteration
            return self._hand_over(item, waited, self.queue.qsize())
        if not self.queue:
            raise StopIteration
        item = self.queue.popleft()
        out = self._hand_over(item, 0.0, len(self.queue))
        self._stage_next()
        return out

    def _hand_over(self, item: _Staged, waited: float, depth: int) -> Any:
        consumer = torch.cuda.current_stream(self.device)
        ready = bool(item.event.query())
        if isinstance(item.batch, dict):
            item.batch["koochak_prefetch_get_wait_s"] = float(waited)
            item.batch["koochak_prefetch_event_ready"] = float(ready)
            item.batch["koochak_prefetch_queue_depth"] = float(depth)
            item.batch["koochak_prefetch_cpu_queue_depth"] = float(item.cpu_queue_depth)
            item.batch["koochak_prefetch_age_s"] = float(max(0.0, time.perf_counter() - item.submitted_at))
            item.batch["koochak_prefetch_prepare_submit_s"] = float(item.submit_cost_s)
        consumer.wait_event(item.event)
        _record_stream(item.batch, consumer)
        return item.batch

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        self._stop.set()
        for name in ("_cuda_worker", "_cpu_worker", "_worker"):
            t = getattr(self, name, None)
            if t is not None:
                t.join(timeout=5.0)


def prefetch(iterable: Iterator[Any], device: torch.device, prefetch: int = 2, *,
             prepare_fn: Optional[BatchPrepareFn] = None, threaded: bool = False,
             pipeline: str = "single") -> Iterator[Any]:
    if getattr(device, "type", "cpu") != "cuda" or prefetch <= 0:
        return iterable
    return CudaPrefetcher(iterable, device=device, prefetch=prefetch, prepare_fn=prepare_fn, threaded=threaded,
                          pipeline=pipeline)


def cycle(iterable: Iterable[Any]) -> Iterator[Any]:
    while True:
        for x in iterable:
            yield x


def take(iterable: Iterable[Any], n: int) -> Iterator[Any]:
    if n <= 0:
        return
    it = iter(iterable)
    for _ in range(n):
        try:
            yield next(it)
        except StopIteration:
            return
