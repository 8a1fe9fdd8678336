"""Datasets written here load in the reference, and both deal shards to workers identically.

The reference is the unmodified package under ``baseline/_ref`` (skipped
when absent), run in a child process. A dataset of tar-encoded samples is
written with this runtime's ``ShardWriter``; the reference's ``load_index``
reads its index and its ``decode_tar_samples`` reads the samples back, and
the reference's ``plan_shards`` deals the shards exactly as this runtime's
does for several seeds, epochs and worker counts.
"""

from __future__ import annotations

import multiprocessing as mp
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
SHIMS = os.path.join(ROOT, "baseline", "shims")

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "koochak")),
                                reason="reference not installed under baseline/_ref")

CASES = [(w, e, s, sh) for w in (1, 3, 5) for e in (0, 2) for s in (0, 11) for sh in (True, False)]


def _reference(root, result):
    import sys

    sys.path[:0] = [REF, SHIMS]
    try:
        from koochak.data.shards import decode_tar_samples, load_index, plan_shards
        from koochak.storage.store import LocalStore

        store = LocalStore(root)
        index = load_index(store, "ds/index.json")
        samples = []
        for shard in index.shards:
            samples += [s["__key__"] for s in decode_tar_samples(store.get(shard.key))]
        plans = {c: [[s.key for s in hand] for hand in plan_shards(index, num_workers=c[0], epoch=c[1], seed=c[2],
                                                                      shuffle=c[3])] for c in CASES}
        result.put(("ok", index.sha256, index.records, samples, plans))
    except Exception as exc:
        import traceback

        result.put(("FAIL", traceback.format_exc()))


def test_reference_reads_dataset_and_deals_the_same(tmp_path):
    from koochak_b200.data.shards import ShardWriter, plan_shards
    from koochak_b200.storage.store import LocalStore

    store = LocalStore(str(tmp_path))
    with ShardWriter(store, "ds", target_bytes=6000, metadata={"source": "synthetic"}) as w:
        for i in range(60):
            w.add({"__key__": f"sample{i:03d}", "txt": f"row {i}".encode() * (i % 7 + 1), "cls": bytes([i % 10])})
    index = w.index
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_reference, args=(str(tmp_path), q))
    p.start()
    p.join(timeout=120)
    got = q.get(timeout=10)
    assert got[0] == "ok", got[1]
    _, sha, records, samples, plans = got
    assert sha == index.sha256 and records == 60 and samples == [f"sample{i:03d}" for i in range(60)]
    for c in CASES:
        mine = [[s.key for s in hand] for hand in plan_shards(index, num_workers=c[0], epoch=c[1], seed=c[2],
                                                               shuffle=c[3])]
        assert mine == plans[c], f"dealing differs for (workers, epoch, seed, shuffle) = {c}"
