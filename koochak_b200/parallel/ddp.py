"""Data-parallel gradient synchronisation, overlapped with backward.

(replaces torch DDP at reference koochak/loop.py:705-723)

``DataParallel`` wraps a module the way ``DistributedDataParallel`` does
(``.module``, ``no_sync()``, parameters broadcast from rank 0 at wrap time,
buffers broadcast before every forward when ``broadcast_buffers``), with its
own bucketing:

* parameters are grouped into buckets of ``bucket_cap_mb`` in reverse
  registration order (the order backward produces gradients), identically on
  every rank;
* a post-accumulate-grad hook copies each finished gradient into its bucket's
  flat fp32 buffer; when a bucket is complete its reduction is launched on a
  dedicated communication stream while backward keeps running;
* at the end of backward the compute stream waits for every bucket and each
  ``param.grad`` becomes a view of the averaged bucket.

Reduction transports (``transport``):

* ``"nccl"`` / ``"gloo"``: one averaging all-reduce per bucket (baseline);
* ``"fused"`` (alias ``"p2p"``): the native single-node path. Buckets live in
  symmetric device memory; one kernel per bucket reduces this rank's shard
  over NVLink (P2P loads or NVSwitch ``multimem``; no NCCL in the data
  path), fused with the GradScaler unscale, the finite flag and per-tensor
  sums of squares, and writes the result back to every rank, with bounded
  cross-GPU flag waits (``koochak_b200/parallel/symm.py``). The gradient gate
  then reads those statistics instead of passing over the gradients again
  (``DataParallel.fused_gate``).

Buckets are launched in index order on every rank, whatever order backward
finishes them in, so every rank issues the same reductions in the same order.
"""

from __future__ import annotations

import contextlib
import os
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist
import torch.nn as nn

__all__ = ["DataParallel", "Bucket"]


class Bucket:
    def __init__(self, index: int, params: List[nn.Parameter], device: torch.device, align: int = 1,
                 allocate: bool = True) -> None:
        self.index = index
        self.params = params
        self.offsets: List[int] = []
        total = 0
        for p in params:
            self.offsets.append(total)
            total += (p.numel() + align - 1) // align * align
        self.numel = total
        # The fused transport replaces this with a view of symmetric memory.
        self.buffer = torch.zeros(total if allocate else 0, device=device, dtype=torch.float32)
        self.pending = 0
        self.work = None
        self.ready_event: Optional[torch.cuda.Event] = None
        self.complete = False

    def view_of(self, i: int) -> torch.Tensor:
        p = self.params[i]
        return self.buffer.narrow(0, self.offsets[i], p.numel()).view_as(p)


class DataParallel(nn.Module):
    def __init__(self, module: nn.Module, *, bucket_cap_mb: float = 25.0, broadcast_buffers: bool = True,
                 transport: str = "auto", process_group=None, find_unused_parameters: bool = False,
                 comm_blocks: Optional[int] = None) -> None:
        super().__init__()
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("DataParallel needs an initialised process group")
        self.module = module
        self.group = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.broadcast_buffers = broadcast_buffers
        self.find_unused_parameters = find_unused_parameters
        self.require_sync = True
        params = [p for p in module.parameters() if p.requires_grad]
        self.device = params[0].device if params else torch.device("cpu")
        backend = str(dist.get_backend(process_group)).lower()
        self.transport = self._pick_transport(transport, backend)
        self._sync_module_states()
        cap = max(1, int(bucket_cap_mb * 1024 * 1024 / 4))
        align, own = (4, False) if self.transport == "fused" else (1, True)
        self.params = params
        self.buckets: List[Bucket] = []
        current: List[nn.Parameter] = []
        size = 0
        for p in reversed(params):
            current.append(p)
            size += p.numel()
            if size >= cap:
                self.buckets.append(Bucket(len(self.buckets), current, self.device, align, own))
                current, size = [], 0
        if current:
            self.buckets.append(Bucket(len(self.buckets), current, self.device, align, own))
        self._where: Dict[int, tuple] = {}
        for b in self.buckets:
            for i, p in enumerate(b.params):
                self._where[id(p)] = (b, i)
        self._comm_stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self._fused = None
        # GradScaler scale (a device scalar, or a callable returning it), applied
        # as 1/scale by the fused path so the reduced gradients come out unscaled.
        self.grad_scale: Optional[torch.Tensor] = None
        self.grad_scale_fn: Optional[Callable[[], Optional[torch.Tensor]]] = None
        self._fused_ready = False
        if self.transport == "fused":
            from .symm import FusedGradReducer

            tid = {id(p): i for i, p in enumerate(params)}
            segments = [[(p.numel(), tid[id(p)]) for p in b.params] for b in self.buckets]
            if comm_blocks is None:  # CTAs per bucket kernel (they share the GPU with the overlapped backward)
                comm_blocks = int(os.environ.get("KOOCHAK_B200_COMM_BLOCKS", 32))
            # CTAs for the reductions that nothing overlaps (after backward).
            self._tail_blocks = max(comm_blocks, int(os.environ.get("KOOCHAK_B200_COMM_TAIL_BLOCKS", 128)))
            self._fused = FusedGradReducer(segments, len(params), self.device, process_group, blocks=comm_blocks)
            for b, buf in zip(self.buckets, self._fused.buffers):
                assert buf.numel() == b.numel
                b.buffer = buf
        self._next_launch = 0
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for p in params]
        self._armed = False
        self._callback_queued = False

    # ------------------------------------------------------------------ setup
    def _pick_transport(self, transport: str, backend: str) -> str:
        t = (transport or "auto").lower()
        if backend != "nccl":
            return "gloo"
        if t == "auto":
            return "nccl"
        if t == "p2p":
            t = "fused"
        if t not in ("nccl", "fused"):
            raise ValueError(f"unknown gradient-sync transport {transport!r}")
        return t

    @torch.no_grad()
    def _sync_module_states(self) -> None:
        for t in list(self.module.parameters()) + list(self.module.buffers()):
            dist.broadcast(t.data, src=0, group=self.group)

    # ------------------------------------------------------------------ forward
    def forward(self, *args, **kwargs):
        if self.broadcast_buffers and self.world > 1:
            with torch.no_grad():
                for b in self.module.buffers():
                    dist.broadcast(b, src=0, group=self.group)
        if torch.is_grad_enabled() and self.require_sync:
            self._arm()
        return self.module(*args, **kwargs)

    @contextlib.contextmanager
    def no_sync(self):
        prev = self.require_sync
        self.require_sync = False
        try:
            yield
        finally:
            self.require_sync = prev

    def _arm(self) -> None:
        self._armed = True
        self._callback_queued = False
        self._fused_ready = False
        self._next_launch = 0
        for b in self.buckets:
            b.pending = len(b.params)
            b.work = None
            b.ready_event = None
            b.complete = False
        if self._fused is not None:
            self._fused.begin_step()

    # ------------------------------------------------------------------ backward
    def _on_grad(self, p: nn.Parameter) -> None:
        if not self._armed:
            return
        if not self._callback_queued:
            torch.autograd.Variable._execution_engine.queue_callback(self._finish)
            self._callback_queued = True
        b, i = self._where[id(p)]
        with torch.no_grad():
            b.view_of(i).copy_(p.grad)
        b.pending -= 1
        if b.pending == 0:
            b.complete = True
            self._launch_ready()

    def _launch_ready(self, tail: bool = False) -> None:
        # Strict index order: the reductions pair up across ranks by sequence.
        # Buckets launched once backward has finished (``tail``), and the last
        # bucket, have no compute left to overlap with: they get the wider
        # grid. Every rank makes the same choice for the same bucket.
        while self._next_launch < len(self.buckets) and self.buckets[self._next_launch].complete:
            b = self.buckets[self._next_launch]
            self._launch(b, wide=tail or b.index == len(self.buckets) - 1)
            self._next_launch += 1

    def _launch(self, b: Bucket, wide: bool = False) -> None:
        if self._comm_stream is None:
            self._reduce_now(b, wide)
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self._comm_stream):
            self._comm_stream.wait_event(ev)
            self._reduce_now(b, wide)
            b.buffer.record_stream(self._comm_stream)
            done = torch.cuda.Event()
            done.record(self._comm_stream)
            b.ready_event = done

    def _reduce_now(self, b: Bucket, wide: bool = False) -> None:
        if self.transport == "fused":
            assert self._fused is not None
            scale = self.grad_scale_fn() if self.grad_scale_fn is not None else self.grad_scale
            self._fused.reduce(b.index, scale, blocks=self._tail_blocks if wide else None)
        elif self.transport == "nccl":
            dist.all_reduce(b.buffer, op=dist.ReduceOp.AVG, group=self.group)
        else:
            dist.all_reduce(b.buffer, group=self.group)
            b.buffer.div_(self.world)

    def _finish(self) -> None:
        # Buckets that never completed (unused parameters) are reduced now so
        # every rank issues the same collectives in the same order.
        for b in self.buckets:
            if b.pending > 0:
                for i, p in enumerate(b.params):
                    if p.grad is None:
                        b.view_of(i).zero_()
                b.pending = 0
                b.complete = True
        self._launch_ready(tail=True)
        cur = torch.cuda.current_stream(self.device) if self._comm_stream is not None else None
        for b in self.buckets:
            if cur is not None and b.ready_event is not None:
                cur.wait_event(b.ready_event)
            for i, p in enumerate(b.params):
                p.grad = b.view_of(i)
        self._fused_ready = self._fused is not None
        self._armed = False

    # ------------------------------------------------------------------ gate
    def fused_gate_available(self) -> bool:
        """True when the last backward was reduced by the fused path (statistics are ready)."""

        return self._fused_ready

    def fused_gate(self, max_norm: Optional[float]) -> torch.Tensor:
        """Device fp32 [4] from the fused statistics: norm, clip coefficient, found_inf, status word.

        The gradients are already averaged and (when ``grad_scale`` was set)
        unscaled; the norm is that of the averaged gradients.
        """

        assert self._fused is not None and self._fused_ready
        return self._fused.gate(max_norm)

    def state_dict(self, *args, **kwargs):
        return {f"module.{k}": v for k, v in self.module.state_dict(*args, **kwargs).items()}

    def load_state_dict(self, state_dict, strict: bool = True):
        stripped = {(k[7:] if k.startswith("module.") else k): v for k, v in state_dict.items()}
        return self.module.load_state_dict(stripped, strict=strict)
