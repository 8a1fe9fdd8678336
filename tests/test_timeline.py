"""The step-timeline analysis: busy time of overlapping kernels, idle gaps and their causes."""

from __future__ import annotations

from types import SimpleNamespace

from koochak_b200.benchmarks.timeline import analyse, report


def _ev(name, start, end, dev):
    return SimpleNamespace(name=name, time_range=SimpleNamespace(start=start, end=end), device_type=dev)


def test_gaps_are_merged_and_attributed():
    events = [
        _ev("gemm", 0, 100, "DeviceType.CUDA"),
        _ev("norm", 50, 120, "DeviceType.CUDA"),        # overlaps the GEMM (another stream)
        _ev("cudaStreamSynchronize", 110, 300, "DeviceType.CPU"),
        _ev("attn", 300, 400, "DeviceType.CUDA"),       # 180 us gap after a host sync
        _ev("cudaLaunchKernel", 395, 440, "DeviceType.CPU"),
        _ev("rope", 450, 460, "DeviceType.CUDA"),       # 50 us gap, launch latency only
        _ev("aten::add", 0, 10, "DeviceType.CPU"),
        _ev("aten::item", 105, 305, "DeviceType.CPU"),  # encloses the synchronisation
        _ev("Optimizer.step#X.step", 0, 400, "DeviceType.CUDA"),  # a GPU user annotation, not a kernel
    ]
    res = analyse(events, gap_us=20.0)
    assert res["window_us"] == 460
    assert res["busy_us"] == 120 + 100 + 10
    assert res["idle_us"] == 460 - 230
    assert res["causes"]["cudaStreamSynchronize in aten::item"] == [1, 180.0]
    assert res["causes"]["host launch latency"] == [1, 50.0]
    assert res["gaps"][0][:2] == (180.0, "cudaStreamSynchronize in aten::item")
    assert res["gaps"][0][2:] == ("norm", "attn")
    assert res["per_kernel"]["gemm"] == [1, 100.0]
    text = report(res, steps=1)
    assert "idle gaps by cause" in text and "cudaStreamSynchronize" in text
