"""Data-parallel gradient synchronisation, overlapped with backward.

(replaces torch DDP at reference koochak/loop.py:705-723)

``DataParallel`` wraps a module the way ``DistributedDataParallel`` does
(``.module``, ``no_sync()``, parameters broadcast from rank 0 at wrap time,
buffers broadcast before every forward when ``broadcast_buffers``), with its
own bucketing:

* parameters are grouped into buckets in reverse registration order (the
  order backward produces gradients), identically on every rank; bucket ``i``
  holds up to ``bucket_caps_mb[min(i, len - 1)]`` MB (torch DDP's
  ``bucket_cap_mb_list`` rule; a single ``bucket_cap_mb`` is a one-entry list);
* a post-accumulate-grad hook copies each finished gradient into its bucket's
  flat fp32 buffer; when a bucket is complete its reduction is launched on a
  dedicated communication stream while backward keeps running;
* at the end of backward the compute stream waits for every bucket and each
  ``param.grad`` becomes a view of its bucket (gradients are always bucket
  views, i.e. torch DDP's ``gradient_as_bucket_view=True``; ``static_graph``
  changes nothing here because buckets are fixed at wrap time).

Reduction transports (``transport``):

* ``"nccl"`` / ``"gloo"``: one averaging all-reduce per bucket (baseline);
* ``"fused"`` (alias ``"p2p"``): the native single-node path. Buckets live in
  symmetric device memory; one kernel per bucket reduces this rank's part
  over NVLink (P2P loads or NVSwitch ``multimem``; no NCCL in the data path),
  fused with the GradScaler unscale, the finite flag and per-tensor sums of
  squares (``koochak_b200/parallel/symm.py``, ``csrc/comm.cu``). The gradient
  gate then reads those statistics instead of passing over the gradients
  again (``DataParallel.fused_gate``).

With the fused transport an optimizer that shards its update can say where
each reduced gradient is needed (``owners``, ``shard_rest``): a parameter
listed in ``owners`` is reduced only into its owner's memory, and with
``shard_rest`` every other parameter is reduce-scattered (rank ``r`` keeps
the reduced values of ``shard_bounds(numel, world, r)``). ``param.grad`` then
holds the averaged gradient only where this rank needs it and this rank's own
local gradient elsewhere; the optimizer (``optim/muon.py``) reads exactly the
averaged parts.

Buckets are launched in index order on every rank, whatever order backward
finishes them in, so every rank issues the same reductions in the same order.
"""

from __future__ import annotations

import contextlib
import os
from typing import Callable, Dict, List, Optional, Sequence, Union

import torch
import torch.distributed as dist
import torch.nn as nn

__all__ = ["DataParallel", "Bucket", "split_buckets"]


def split_buckets(numels: Sequence[int], caps: Sequence[int]) -> List[List[int]]:
    """Group parameter indices (already in gradient order) into buckets.

    Bucket ``i`` is closed as soon as it holds at least ``caps[min(i, len(caps) - 1)]``
    elements, so one large tensor always forms a bucket of its own.
    """

    out: List[List[int]] = []
    cur: List[int] = []
    size = 0
    for i, n in enumerate(numels):
        cur.append(i)
        size += int(n)
        if size >= caps[min(len(out), len(caps) - 1)]:
            out.append(cur)
            cur, size = [], 0
    if cur:
        out.append(cur)
    return out


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
        self.ready_event: Optional[torch.cuda.Event] = None
        self.complete = False

    def view_of(self, i: int) -> torch.Tensor:
        p = self.params[i]
        return self.buffer.narrow(0, self.offsets[i], p.numel()).view_as(p)


class DataParallel(nn.Module):
    def __init__(self, module: nn.Module, *, bucket_cap_mb: Union[float, Sequence[float]] = 25.0,
                 broadcast_buffers: bool = True, transport: str = "auto", process_group=None,
                 find_unused_parameters: bool = False, comm_blocks: Optional[int] = None,
                 owners: Optional[Dict[int, int]] = None, shard_rest: bool = False,
                 reserve_sms: Optional[int] = None) -> None:
        """``owners`` maps ``id(param)`` to the rank that alone needs its reduced gradient (fused transport only).

        ``reserve_sms``: while reductions overlap backward, keep that many SMs
        free of the persistent GEMM / attention grids and run the reductions on
        them (fused transport only). ``None`` picks it from
        ``KOOCHAK_B200_COMM_RESERVE_SMS``, else 24 when the gradients exceed
        1 GiB (long reductions that would otherwise wait for whole persistent
        grids to drain) and 0 below that.
        """

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
        caps_mb = [float(bucket_cap_mb)] if isinstance(bucket_cap_mb, (int, float)) else [float(c) for c in bucket_cap_mb]
        if not caps_mb or any(c <= 0 for c in caps_mb):
            raise ValueError("bucket caps must be positive")
        caps = [max(1, int(c * 1024 * 1024 / 4)) for c in caps_mb]
        align, own = (4, False) if self.transport == "fused" else (1, True)
        self.params = params
        order = list(reversed(params))
        self.buckets: List[Bucket] = [
            Bucket(i, [order[j] for j in idx], self.device, align, own)
            for i, idx in enumerate(split_buckets([p.numel() for p in order], caps))
        ]
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
        self._reserve = 0
        self._reserving = False
        self.owners: Dict[int, int] = {}
        self.shard_rest = False
        if self.transport == "fused":
            from .symm import FusedGradReducer

            tid = {id(p): i for i, p in enumerate(params)}
            self.owners = {k: int(v) for k, v in (owners or {}).items() if k in tid}
            self.shard_rest = bool(shard_rest)
            segments = [[(p.numel(), tid[id(p)]) for p in b.params] for b in self.buckets]
            if comm_blocks is None:  # CTAs per bucket kernel (they share the GPU with the overlapped backward)
                comm_blocks = int(os.environ.get("KOOCHAK_B200_COMM_BLOCKS", 32))
            # CTAs for the reductions that nothing overlaps (after backward).
            self._tail_blocks = max(comm_blocks, int(os.environ.get("KOOCHAK_B200_COMM_TAIL_BLOCKS", 128)))
            self._fused = FusedGradReducer(segments, len(params), self.device, process_group, blocks=comm_blocks,
                                           owner_of={tid[k]: r for k, r in self.owners.items()},
                                           shard_rest=self.shard_rest)
            for b, buf in zip(self.buckets, self._fused.buffers):
                assert buf.numel() == b.numel
                b.buffer = buf
            if reserve_sms is None:
                env = os.environ.get("KOOCHAK_B200_COMM_RESERVE_SMS")
                total = 4 * sum(b.numel for b in self.buckets)
                reserve_sms = int(env) if env is not None else (24 if total > (1 << 30) else 0)
            self._reserve = max(0, int(reserve_sms))
        elif owners or shard_rest:
            raise ValueError("owners / shard_rest need the fused transport")
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

    @property
    def sharded(self) -> bool:
        """True when some reduced gradients live only on the rank that owns them."""

        return bool(self.owners) or self.shard_rest

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

    def _set_reserve(self, on: bool) -> None:
        if self._reserve and on != self._reserving:
            from ..ops._ext import native

            native().set_sm_reserve(self._reserve if on else 0)
            self._reserving = on

    def _arm(self) -> None:
        self._set_reserve(False)
        if self._fused is not None and self._fused_ready:
            # The previous synchronised backward was never gated: close its
            # reductions on every rank before the buckets are written again.
            self._fused.seal_gate(None)
        self._armed = True
        self._callback_queued = False
        self._fused_ready = False
        self._next_launch = 0
        for b in self.buckets:
            b.pending = len(b.params)
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
        # Strict index order: every rank issues the same reductions in the same
        # sequence. Buckets launched once backward has finished (``tail``), and
        # the last bucket, have no compute left to overlap with and get the
        # wider grid; the fused kernels' arrival protocol does not need the
        # grids of different ranks to agree.
        while self._next_launch < len(self.buckets) and self.buckets[self._next_launch].complete:
            b = self.buckets[self._next_launch]
            wide = tail or b.index == len(self.buckets) - 1
            if not wide:
                self._set_reserve(True)
            self._launch(b, wide=wide)
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
            blocks = self._tail_blocks if wide else (self._reserve or None)
            self._fused.reduce(b.index, scale, blocks=blocks)
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
        self._set_reserve(False)
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

        Waits (on the device, bounded) for every rank's last bucket kernel
        first. The gradients are averaged and (when ``grad_scale`` was set)
        unscaled; the norm is that of the averaged gradients.
        """

        assert self._fused is not None and self._fused_ready
        self._fused_ready = False
        return self._fused.seal_gate(max_norm)

    def state_dict(self, *args, **kwargs):
        return {f"module.{k}": v for k, v in self.module.state_dict(*args, **kwargs).items()}

    def load_state_dict(self, state_dict, strict: bool = True):
        stripped = {(k[7:] if k.startswith("module.") else k): v for k, v in state_dict.items()}
        return self.module.load_state_dict(stripped, strict=strict)
