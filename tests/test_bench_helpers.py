"""Host-side helpers of the benchmark and the Muon batching rule (no GPU)."""

from __future__ import annotations

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _sample(t, mhz, cap):
    return (t, float(mhz), 1965.0, frozenset({"sw_power_cap"}) if cap else frozenset())


def test_clock_sampler_keeps_the_timed_window():
    import bench

    c = bench.ClockSampler(0)
    c.samples = [_sample(1.0, 1100, False), _sample(2.2, 1800, True), _sample(2.6, 1700, True),
                 _sample(4.0, 600, False)]
    out = c.stop(2.0, 3.0)
    assert out["samples"] == 2 and out["sm_mhz"] == 1750.0 and out["window"] == "timed"
    assert out["reasons"] == ["sw_power_cap"] and out["sm_max_mhz"] == 1965.0


def test_clock_sampler_falls_back_to_the_end_of_warmup():
    import bench

    c = bench.ClockSampler(0)
    c.samples = [_sample(0.5, 900, False), _sample(1.7, 1850, True)]
    out = c.stop(2.0, 2.1)  # timed region shorter than the sampling period
    assert out["samples"] == 1 and out["sm_mhz"] == 1850.0 and out["window"] == "last second of warm-up"


def test_transposed_shape_buckets_share_one_newton_schulz_batch():
    from koochak_b200.optim.muon import _batches, _muon_buckets

    ps = [torch.nn.Parameter(torch.zeros(s)) for s in [(768, 3072), (3072, 768), (768, 768), (3072, 768), (64, 96)]]
    buckets = _muon_buckets(ps)
    batches = _batches({k: [ps[i] for i in idx] for k, idx in buckets.items()})
    shapes = sorted(sorted((R, C, len(q)) for R, C, q in parts) for parts in batches)
    assert shapes == [[(64, 96, 1)], [(768, 768, 1)], [(768, 3072, 1), (3072, 768, 2)]]
