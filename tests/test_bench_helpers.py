"""Host-side helpers of the benchmark and the Muon batching rule (no GPU)."""

from __future__ import annotations

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

LINE = "0, {mhz}, 1965, 900.0, 0x4, Not Active, Not Active, Not Active, {cap}"


def test_clock_sampler_keeps_the_timed_window():
    import bench

    c = bench.ClockSampler(0)
    c.lines = [(1.0, LINE.format(mhz=1100, cap="Not Active")), (2.2, LINE.format(mhz=1800, cap="Active")),
               (2.6, LINE.format(mhz=1700, cap="Active")), (4.0, LINE.format(mhz=600, cap="Not Active"))]
    out = c.stop(2.0, 3.0)
    assert out["samples"] == 2 and out["sm_mhz"] == 1750.0 and out["window"] == "timed"
    assert out["reasons"] == ["sw_power_cap"] and out["sm_max_mhz"] == 1965.0


def test_clock_sampler_falls_back_to_the_end_of_warmup():
    import bench

    c = bench.ClockSampler(0)
    c.lines = [(0.5, LINE.format(mhz=900, cap="Not Active")), (1.7, LINE.format(mhz=1850, cap="Active"))]
    out = c.stop(2.0, 2.1)  # timed region shorter than the sampling period
    assert out["samples"] == 1 and out["sm_mhz"] == 1850.0 and out["window"] == "last second of warm-up"


def test_transposed_shape_buckets_share_one_newton_schulz_batch():
    from koochak_b200.optim.muon import _batches, _muon_buckets

    ps = [torch.nn.Parameter(torch.zeros(s)) for s in [(768, 3072), (3072, 768), (768, 768), (3072, 768), (64, 96)]]
    buckets = _muon_buckets(ps)
    batches = _batches({k: [ps[i] for i in idx] for k, idx in buckets.items()})
    shapes = sorted(sorted((R, C, len(q)) for R, C, q in parts) for parts in batches)
    assert shapes == [[(64, 96, 1)], [(768, 768, 1)], [(768, 3072, 1), (3072, 768, 2)]]
