"""CUDA prefetcher: every mode delivers every batch, in order, on the consumer's stream.

Inline, one worker thread and the two-stage (fetch thread + staging thread)
pipeline each move dict batches from pinned host memory to the GPU with an
optional ``prepare_fn`` on the side stream; an exception inside the source
iterator reaches the consumer. On CPU only the pass-through and helpers run.
"""

from __future__ import annotations

import pytest
import torch

from koochak_b200.data.iterable import CudaPrefetcher, cycle, prefetch, take, to_device


def test_helpers_and_cpu_passthrough():
    src = [1, 2, 3]
    assert prefetch(src, torch.device("cpu"), 2) is src
    assert list(take(cycle([1, 2]), 5)) == [1, 2, 1, 2, 1]
    assert list(take([1], 3)) == [1]
    nested = {"a": torch.ones(2), "b": [torch.zeros(1), (torch.ones(1), "x")]}
    out = to_device(nested, torch.device("cpu"))
    assert isinstance(out["b"][1], tuple) and out["b"][1][1] == "x"


def _batches(n):
    return [{"x": torch.full((4, 8), float(i)).pin_memory(), "i": torch.tensor([i])} for i in range(n)]


@pytest.mark.gpu
@pytest.mark.parametrize("threaded,pipeline", [(False, "single"), (True, "single"), (True, "two_stage")])
def test_prefetch_modes_deliver_in_order(threaded, pipeline):
    dev = torch.device("cuda", 0)

    def prep(b):
        b["y"] = b["x"] * 2
        return b

    pf = CudaPrefetcher(iter(_batches(7)), dev, prefetch=3, prepare_fn=prep, threaded=threaded, pipeline=pipeline)
    seen = []
    for b in pf:
        assert b["x"].is_cuda and b["y"].is_cuda
        assert float(b["y"][0, 0]) == 2.0 * float(b["i"][0])
        assert "koochak_prefetch_age_s" in b and "koochak_prefetch_get_wait_s" in b
        seen.append(int(b["i"][0]))
    pf.close()
    assert seen == list(range(7))


@pytest.mark.gpu
@pytest.mark.parametrize("pipeline", ["single", "two_stage"])
def test_prefetch_worker_error_reaches_consumer(pipeline):
    def source():
        yield {"x": torch.ones(2)}
        raise KeyError("broken batch")

    pf = CudaPrefetcher(source(), torch.device("cuda", 0), prefetch=2, threaded=True, pipeline=pipeline)
    next(pf)
    with pytest.raises(KeyError):
        next(pf)
    pf.close()
