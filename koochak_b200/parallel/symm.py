"""Symmetric device memory and the fused gradient synchronisation built on it.

(replaces the NCCL bucket all-reduce of torch DDP used at reference
koochak/loop.py:705-723, and the unscale / finite check / norm pass of
koochak/loop.py:1612-1637 and koochak/optim/grad_clip.py:47-73)

``SymmetricWorkspace`` allocates one buffer per rank through PyTorch's
symmetric-memory allocator (same size and layout on every GPU of the node,
each rank's buffer mapped into every peer) and, where the NVSwitch supports
it, a multicast mapping of the same buffer. Only the addresses come from
PyTorch: the kernels that read and write peers are this package's own
(``koochak_b200/csrc/comm.cu``).

``FusedGradReducer`` lays the data-parallel buckets out inside such a
workspace. For bucket ``b`` it launches one kernel that waits (bounded) until
every rank has produced bucket ``b`` and then, for each chunk of this rank's
part of the bucket, sums the ranks' values over NVLink (P2P loads, or
``multimem.ld_reduce`` through the switch), multiplies by ``inv_scale / W``,
checks finiteness, accumulates per-tensor sums of squares into every rank's
statistics, and stores the result either into every rank (a replicated
tensor: all-reduce) or into this rank only (a tensor whose owner alone needs
the reduced gradient: a Muon matrix, or this rank's shard of a tensor whose
optimizer update is sharded). Which rank handles which part is fixed by
``plan_bucket_chunks``. After the last bucket, ``seal_gate`` waits for every
rank's bucket kernels and forms the clip statistics in one small kernel.
"""

from __future__ import annotations

import os
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

__all__ = ["SymmetricWorkspace", "FusedGradReducer", "SymmetricParamSlab", "plan_chunks", "plan_bucket_chunks",
           "shard_bounds"]

_FLAG_BYTES = 256  # [max ranks] u32 arrival slots, padded to the allocation alignment
_ALIGN = 256


def _align(n: int, a: int = _ALIGN) -> int:
    return (n + a - 1) // a * a


def shard_bounds(numel: int, world: int, rank: int, align: int = 4) -> Tuple[int, int]:
    """[lo, hi) of ``rank``'s shard of ``numel`` elements; boundaries are multiples of ``align``."""

    per = (numel + world - 1) // world
    per = (per + align - 1) // align * align
    lo = min(numel, rank * per)
    hi = min(numel, lo + per)
    return lo, hi


def plan_chunks(segments: Sequence[Tuple[int, int, int]], lo: int, hi: int, max_chunk: int = 32768) -> List[Tuple[int, int, int]]:
    """Split ``[lo, hi)`` of a bucket into (start, length, tensor id) pieces.

    ``segments`` are (offset, numel, tensor id) of the tensors in the bucket
    (offsets multiples of 4). Pieces never cross a tensor, start on a multiple
    of 4 elements and hold at most ``max_chunk`` elements.
    """

    out: List[Tuple[int, int, int]] = []
    for off, n, tid in segments:
        a, b = max(lo, off), min(hi, off + n)
        while a < b:
            step = min(max_chunk, b - a)
            if a + step < b:
                step = max(4, step // 4 * 4)
            out.append((a, step, tid))
            a += step
    return out


MODE_ALL = 0    # reduced value written to every rank
MODE_LOCAL = 1  # reduced value written to the reducing rank only


def plan_bucket_chunks(layout: Sequence[Tuple[int, int, int]], world: int, rank: int,
                       owner_of: Optional[Dict[int, int]] = None, shard_rest: bool = False,
                       max_chunk: int = 32768) -> List[Tuple[int, int, int, int]]:
    """This rank's (start, length, tensor id, mode) pieces of one bucket.

    ``layout`` lists (offset, numel, tensor id) of the bucket's tensors.
    A tensor in ``owner_of`` is reduced whole by its owner, into the owner's
    memory only. Every other tensor is split evenly over the ranks
    (``shard_bounds``); each rank reduces its piece and writes it to every
    rank, or, with ``shard_rest``, to itself only (a reduce-scatter whose
    shards are the per-tensor ``shard_bounds``).
    """

    owner_of = owner_of or {}
    out: List[Tuple[int, int, int, int]] = []
    for off, n, tid in layout:
        if tid in owner_of:
            if owner_of[tid] == rank:
                out += [(a, ln, t, MODE_LOCAL) for a, ln, t in plan_chunks([(off, n, tid)], off, off + n, max_chunk)]
            continue
        lo, hi = shard_bounds(n, world, rank)
        mode = MODE_LOCAL if shard_rest else MODE_ALL
        out += [(a, ln, t, mode) for a, ln, t in plan_chunks([(off, n, tid)], off + lo, off + hi, max_chunk)]
    return out


class SymmetricWorkspace:
    """One symmetric buffer per rank (and its multicast mapping when available)."""

    def __init__(self, nbytes: int, device: torch.device, group=None, *, use_multicast: Optional[bool] = None) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = device
        self.nbytes = _align(nbytes)
        self.tensor = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.handle = symm_mem.rendezvous(self.tensor, self.group)
        own = int(self.handle.buffer_ptrs[self.rank])
        offset = self.tensor.data_ptr() - own
        self.bases = [int(p) + offset for p in self.handle.buffer_ptrs]
        mc = 0
        if use_multicast is None:
            use_multicast = os.environ.get("KOOCHAK_B200_MULTIMEM", "1") != "0"
        if use_multicast and self.world > 1:
            try:
                if symm_mem._SymmetricMemory.has_multicast_support(symm_mem.DeviceType.CUDA, device.index or 0):
                    mc = int(self.handle.multicast_ptr)
            except Exception:  # no NVSwitch multicast here: plain peer loads and stores
                mc = 0
        self.mc_base = mc + offset if mc else 0

    def view(self, offset: int, numel: int, dtype: torch.dtype) -> torch.Tensor:
        size = numel * torch.empty((), dtype=dtype).element_size()
        return self.tensor.narrow(0, offset, size).view(dtype)


class FusedGradReducer:
    """Bucketed, fused gradient reduction over a symmetric workspace."""

    def __init__(self, bucket_segments: Sequence[Sequence[Tuple[int, int]]], n_tensors: int, device: torch.device,
                 group=None, *, blocks: int = 32, timeout_s: Optional[float] = None,
                 use_multicast: Optional[bool] = None, owner_of: Optional[Dict[int, int]] = None,
                 shard_rest: bool = False) -> None:
        """``bucket_segments[b]`` lists (numel, tensor id) of bucket ``b``'s tensors, in layout order.

        ``owner_of`` (tensor id -> rank) and ``shard_rest`` select where each
        reduced value goes (``plan_bucket_chunks``); by default every tensor
        is all-reduced.
        """

        from ..ops._ext import native

        self._C = native()
        self.n_tensors = int(n_tensors)
        self.blocks = int(blocks)
        self.timeout_s = float(timeout_s if timeout_s is not None else os.environ.get("KOOCHAK_B200_COMM_TIMEOUT_S", 300))
        self.owner_of = dict(owner_of or {})
        self.shard_rest = bool(shard_rest)
        stats_bytes = _align(4 * (self.n_tensors + 1))
        self.flags_off = 0
        self.stats_off = [_FLAG_BYTES, _FLAG_BYTES + stats_bytes]
        off = _align(_FLAG_BYTES + 2 * stats_bytes)
        self.bucket_off: List[int] = []
        self.bucket_numel: List[int] = []
        self.layouts: List[List[Tuple[int, int, int]]] = []  # (offset, numel, tensor id)
        for segs in bucket_segments:
            layout, cur = [], 0
            for numel, tid in segs:
                layout.append((cur, int(numel), int(tid)))
                cur += (int(numel) + 3) // 4 * 4
            self.layouts.append(layout)
            self.bucket_off.append(off)
            self.bucket_numel.append(cur)
            off = _align(off + 4 * cur)
        self.ws = SymmetricWorkspace(off, device, group, use_multicast=use_multicast)
        self.world, self.rank = self.ws.world, self.ws.rank
        self.buffers = [self.ws.view(o, n, torch.float32) for o, n in zip(self.bucket_off, self.bucket_numel)]
        self.chunks: List[torch.Tensor] = []
        self.work: List[int] = []  # elements this rank reduces per bucket
        for layout in self.layouts:
            rows = plan_bucket_chunks(layout, self.world, self.rank, self.owner_of, self.shard_rest)
            self.work.append(sum(r[1] for r in rows))
            rows = rows or [(0, 0, 0, MODE_ALL)]
            self.chunks.append(torch.tensor(rows, dtype=torch.int64, device=device))
        self.stats = [self.ws.view(o, self.n_tensors + 1, torch.float32) for o in self.stats_off]
        self.parity = 0
        self.epoch = 1
        with torch.no_grad():
            self.ws.tensor.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=self.ws.group)
        self.barrier()  # every rank's flags are zero and mapped

    # ---------------------------------------------------------------- per step
    def begin_step(self) -> None:
        """Select and clear this step's statistics copy (call on the compute stream before backward)."""

        self.parity ^= 1
        self.stats[self.parity].zero_()

    def current_stats(self) -> torch.Tensor:
        return self.stats[self.parity]

    def _next_epoch(self) -> int:
        e = self.epoch
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        return e

    def reduce(self, b: int, scale: Optional[torch.Tensor] = None, blocks: Optional[int] = None) -> None:
        """Reduce bucket ``b`` (average, unscale, statistics) on the current stream.

        ``blocks`` overrides the grid size of this launch (at most 148); the
        arrival protocol does not need it to agree across ranks.
        """

        nb = min(int(blocks), 148) if blocks else self.blocks
        self._C.comm_grad_sync(self.ws.bases, self.ws.mc_base, self.flags_off, self.stats_off[self.parity],
                               self.bucket_off[b], self.chunks[b], self.n_tensors, self.rank, self._next_epoch(),
                               scale, nb, self.timeout_s, self.ws.nbytes)

    def barrier(self) -> None:
        self._C.comm_barrier(self.ws.bases, self.flags_off, self.rank, self._next_epoch(), 1, self.timeout_s,
                             self.ws.device.index or 0)

    def seal_gate(self, max_norm: Optional[float]) -> torch.Tensor:
        """After the last bucket: wait for every rank, then device fp32 [4] = norm, clip coefficient, found_inf, status."""

        out = torch.empty(4, device=self.ws.device, dtype=torch.float32)
        self._C.comm_gate_seal(self.ws.bases, self.flags_off, self.stats_off[self.parity], self.n_tensors, self.rank,
                               self._next_epoch(), self.timeout_s, float(max_norm or 0.0), max_norm is not None, out)
        return out

    def gate(self, max_norm: Optional[float]) -> torch.Tensor:
        """Device fp32 [4] from this rank's statistics (no wait for peers)."""

        out = torch.empty(4, device=self.ws.device, dtype=torch.float32)
        self._C.gate_from_stats(self.current_stats(), self.n_tensors, float(max_norm or 0.0), max_norm is not None, out)
        return out


class SymmetricParamSlab:
    """fp32 parameters stored in symmetric memory, so an owner can write its update into every rank's copy.

    Each listed parameter's storage is moved (``p.data = view``) into one
    symmetric buffer laid out identically on every rank, values preserved.
    The sharded Muon step (``optim/muon.py``) then has the owning rank of
    each matrix store its updated value into all ranks' slabs from inside the
    update kernel (``csrc/muon_gather.cu``), replacing the per-bucket
    all-gather; ``barrier()`` (bounded, cross-GPU) is the point after which
    every rank may read the new values.
    """

    def __init__(self, params: Sequence[torch.Tensor], device: torch.device, group=None, *,
                 timeout_s: Optional[float] = None, use_multicast: Optional[bool] = None) -> None:
        from ..ops._ext import native

        self._C = native()
        self.params = list(params)
        self.timeout_s = float(timeout_s if timeout_s is not None else os.environ.get("KOOCHAK_B200_COMM_TIMEOUT_S", 300))
        offsets, off = [], _FLAG_BYTES
        for p in self.params:
            offsets.append(off)
            off = _align(off + 4 * p.numel())
        self.ws = SymmetricWorkspace(off, device, group, use_multicast=use_multicast)
        self.world, self.rank = self.ws.world, self.ws.rank
        self.epoch = 1
        with torch.no_grad():
            self.ws.tensor.narrow(0, 0, _FLAG_BYTES).zero_()
            for p, o in zip(self.params, offsets):
                view = self.ws.view(o, p.numel(), torch.float32).view(p.shape)
                view.copy_(p.detach())
                p.data = view
                if getattr(p, "_kb_shadow", None) is not None:
                    p._kb_shadow_version = -1  # type: ignore[attr-defined]
        torch.cuda.synchronize(device)
        dist.barrier(group=self.ws.group)
        self.barrier()

    def holds(self, params: Sequence[torch.Tensor]) -> bool:
        """True while ``params`` are exactly this slab's parameters and still stored in it."""

        if len(params) != len(self.params) or any(a is not b for a, b in zip(params, self.params)):
            return False
        lo = self.ws.tensor.data_ptr()
        hi = lo + self.ws.nbytes
        return all(lo <= p.data_ptr() < hi for p in self.params)

    def barrier(self) -> None:
        e = self.epoch
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        self._C.comm_barrier(self.ws.bases, 0, self.rank, e, 1, self.timeout_s, self.ws.device.index or 0)
