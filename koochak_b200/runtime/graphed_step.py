"""Forward and backward of a training step captured once as a CUDA graph and replayed.

A single-GPU step of the benchmark models launches a few hundred kernels for
forward and backward; on B200 the host needs about as long to enqueue them
as the GPU needs to run them, so the GPU idles wherever the host has a burst
of work (the optimizer's preparation, logging). Captured into one CUDA graph,
forward and backward become one launch and the host runs ahead.

``GraphedStep`` (``train.cuda_graph_step: true``) runs the first
``warmup`` updates eagerly (lazy initialisation of the native library, the
allocator and the autograd graph happens there), captures the next one --
``step_fn`` on static copies of the batch tensors, the loss scaling and
``backward`` -- and replays the graph from then on. The gate, the optimizer,
the EMA and everything else of the update stay eager. Preconditions, checked
where they can be:

* one process (a data-parallel wrapper reduces gradients from hooks, which
  a replay does not run), one micro-batch per update (``grad_accum == 1``),
  a CUDA device;
* every batch a mapping of tensors with the captured shapes and dtypes (a
  batch that differs runs eagerly);
* ``step_fn`` behaves the same on every step: what it computes must not
  depend on ``ctx`` or on host state (the forced-overflow benchmark step, for
  instance, must run eagerly);
* the model keeps its 16-bit weight copies in place (``LowPrecisionShadows``);
  stale copies are refreshed eagerly before every replay, since the replay
  skips the forward's Python code.

Gradients: the captured backward returns them (``torch.autograd.grad``
over the parameters) into buffers of the graph's memory pool; every replay
rewrites them, and after each replay those tensors are set as ``.grad``.
Kernels of this library that the graph launches are added to the library's
launch counter on every replay.
"""

from __future__ import annotations

import contextlib
from typing import Any, Callable, Dict, List, Mapping, Optional, Tuple

import torch

__all__ = ["GraphedStep"]


def _signature(batch: Any) -> Optional[Tuple]:
    if not isinstance(batch, Mapping):
        return None
    sig = []
    for k in sorted(batch, key=str):
        v = batch[k]
        if not isinstance(v, torch.Tensor):
            return None
        sig.append((str(k), tuple(v.shape), v.dtype, v.device))
    return tuple(sig)


class GraphedStep:
    def __init__(self, model: torch.nn.Module, *, warmup: int = 3) -> None:
        self.model = model
        self.warmup = max(1, int(warmup))
        self.eager_steps = 0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.sig: Optional[Tuple] = None
        self.static: Dict[str, torch.Tensor] = {}
        self.out: Optional[Mapping[str, Any]] = None
        self.loss: Optional[torch.Tensor] = None
        self.grads: List[Tuple[torch.nn.Parameter, torch.Tensor]] = []
        self.kernels_per_replay = 0
        self.disabled = False
        self.stream: Optional[torch.cuda.Stream] = None

    # ------------------------------------------------------------------ helpers
    def _refresh_shadows(self) -> None:
        for m in self.model.modules():
            shadows = getattr(m, "_shadows", None)
            refresh = getattr(shadows, "refresh", None)
            if callable(refresh):
                refresh()

    def _launch_count(self) -> int:
        try:
            from ..ops._ext import native

            return int(native().launch_count())
        except ImportError:
            return 0

    # ------------------------------------------------------------------ API
    def wants(self, batch: Any) -> bool:
        """Whether this update goes through the graph (capture or replay) instead of the eager path."""

        if self.disabled:
            return False
        if self.graph is None:
            return self.eager_steps >= self.warmup and _signature(batch) is not None
        return _signature(batch) == self.sig

    def note_eager(self) -> None:
        self.eager_steps += 1

    @contextlib.contextmanager
    def on_side_stream(self):
        """Run a micro-step's forward and backward on the graph's stream, ordered after earlier work.

        The parameters' gradient-accumulation nodes are created on the stream
        current at their first use and live as long as the module; running
        the eager updates and the capture on one stream keeps them on it (a
        capture that met nodes of the default stream would fail).
        """

        if self.stream is None:
            self.stream = torch.cuda.Stream()
        cur = torch.cuda.current_stream()
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            yield
        cur.wait_stream(self.stream)

    def run(self, batch: Mapping[str, torch.Tensor],
            forward: Callable[[Mapping[str, torch.Tensor]], Tuple[Mapping[str, Any], torch.Tensor, torch.Tensor]]
            ) -> Tuple[Mapping[str, Any], torch.Tensor]:
        """Forward and backward of ``batch``; returns (step_fn's output, the micro-step loss).

        ``forward(batch)`` returns (step_fn's output, the micro-step loss, the
        loss to differentiate -- the scaled one under a GradScaler).
        """

        if self.graph is None:
            self._capture(batch, forward)  # counted once, at capture
        else:
            for k, v in batch.items():
                self.static[str(k)].copy_(v, non_blocking=True)
            self._refresh_shadows()
            self.graph.replay()
            if self.kernels_per_replay:
                from ..ops._ext import native

                native().add_launches(self.kernels_per_replay)
        for p, g in self.grads:
            p.grad = g
        assert self.out is not None and self.loss is not None
        return self.out, self.loss

    def _capture(self, batch, forward) -> None:
        self.sig = _signature(batch)
        self.static = {str(k): v.detach().clone() for k, v in batch.items()}
        params = [p for p in self.model.parameters() if p.requires_grad]
        for p in params:
            p.grad = None
        self._refresh_shadows()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        before = self._launch_count()
        try:
            with torch.cuda.graph(graph, stream=self.stream, capture_error_mode="thread_local"):
                out, loss, scaled = forward(self.static)
                # Gradients as outputs of the captured backward, in buffers of the graph's pool.
                grads = torch.autograd.grad(scaled, params, allow_unused=True)
        except Exception:
            self.disabled = True
            raise
        self.kernels_per_replay = self._launch_count() - before
        self.graph = graph
        self.out, self.loss = out, loss
        self.grads = [(p, g) for p, g in zip(params, grads) if g is not None]
        graph.replay()  # capture records the kernels without running them
