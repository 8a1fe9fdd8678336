"""Dataset shards, collections, transfer, archive / pull / verify (CPU, local stores)."""

from __future__ import annotations

import os

import pytest

from koochak_b200.storage.store import LocalStore


def test_shard_writer_index_and_plan(tmp_path):
    from koochak_b200.data.shards import (TAR, ShardWriter, assign_shards, decode_tar_samples, load_index,
                                          plan_shards, read_shard)

    store = LocalStore(str(tmp_path / "ds"))
    with ShardWriter(store, "train", target_bytes=4096, metadata={"name": "toy"}) as w:
        for i in range(40):
            w.add({"__key__": f"s{i:04d}", "txt": f"record {i}".encode(), "cls": str(i % 3).encode()})
    idx = load_index(store, "train/index.json")
    assert idx.records == 40 and len(idx.shards) > 2 and idx.metadata["name"] == "toy"
    got = [s for sh in idx.shards for s in TAR.decode(read_shard(store, sh))]
    assert [g["__key__"] for g in got] == [f"s{i:04d}" for i in range(40)]
    assert got[7]["txt"] == b"record 7"
    plan = plan_shards(idx, num_workers=2, epoch=1, seed=3)
    assert sorted(s.key for w in plan for s in w) == sorted(s.key for s in idx.shards)
    assert assign_shards(idx, worker=1, num_workers=2, epoch=1, seed=3) == plan[1]
    assert plan_shards(idx, num_workers=2, epoch=1, seed=3) == plan  # a pure function of its arguments
    # Rebuilding the same dataset is accepted (identical bytes); different content is refused.
    with ShardWriter(store, "train", target_bytes=4096, metadata={"name": "toy"}) as w:
        for i in range(40):
            w.add({"__key__": f"s{i:04d}", "txt": f"record {i}".encode(), "cls": str(i % 3).encode()})
    with pytest.raises(FileExistsError):
        with ShardWriter(store, "train", target_bytes=4096) as w:
            w.add({"__key__": "x", "txt": b"different"})
    assert list(decode_tar_samples(read_shard(store, idx.shards[0])))[0]["__key__"] == "s0000"


def _tree(root):
    files = {"a/x.txt": b"x" * 10, "a/y.txt": b"yy", "b/z.bin": os.urandom(5000), "big.bin": os.urandom(70000)}
    for rel, data in files.items():
        p = root / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_bytes(data)
    return files


def test_archive_pull_verify_resume(tmp_path):
    from koochak_b200.storage.archive import archive, pull, verify
    from koochak_b200.storage.collection import load_collection

    src = tmp_path / "src"
    files = _tree(src)
    store = LocalStore(str(tmp_path / "arch"))
    rep = archive(str(src), store, pack_bytes=8192, object_bytes=65536, metadata={"v": 1})
    col = load_collection(store)
    assert {f.path for f in col.files} == set(files)
    assert any(f.object for f in col.files) and any(f.pack is not None for f in col.files)
    assert verify(store, deep=True).ok
    again = archive(str(src), store, pack_bytes=8192, object_bytes=65536, metadata={"v": 1})
    assert again.packs_written == 0 and again.packs_reused == rep.packs_written
    dst = LocalStore(str(tmp_path / "out"))
    r = pull(store, dst, patterns=["a/*"])
    assert r.files == 2 and (tmp_path / "out" / "a" / "y.txt").read_bytes() == b"yy"
    r = pull(store, dst)
    assert r.skipped == 2 and (tmp_path / "out" / "big.bin").read_bytes() == files["big.bin"]
    assert os.stat(tmp_path / "out" / "b" / "z.bin").st_mtime_ns == os.stat(src / "b" / "z.bin").st_mtime_ns


def test_copy_objects_resumes_and_checks(tmp_path):
    import hashlib

    from koochak_b200.storage.transfer import TransferItem, copy_objects

    a, b = LocalStore(str(tmp_path / "a")), LocalStore(str(tmp_path / "b"))
    blobs = {f"k{i}": os.urandom(1000 * (i + 1)) for i in range(5)}
    for k, v in blobs.items():
        a.put(k, v)
    items = [TransferItem(k, "c/" + k, len(v), hashlib.sha256(v).hexdigest()) for k, v in blobs.items()]
    rep = copy_objects(a, b, items, streams=3, range_streams=2, part_bytes=700)
    assert rep.copied == 5 and b.get("c/k3") == blobs["k3"]
    rep = copy_objects(a, b, items)
    assert rep.skipped == 5 and rep.copied == 0
    bad = [TransferItem("k0", "d/k0", 1000, "0" * 64)]
    with pytest.raises(ValueError):
        copy_objects(a, b, bad)
    assert b.stat("d/k0") is None


def test_packed_groups_stream_and_data_cli(tmp_path, capsys):
    from koochak_b200.data.__main__ import main as data_main
    from koochak_b200.data.packed import GroupStream, PackCache, PackedGroups

    src = tmp_path / "src"
    rows = ["path,group,order"]
    for g in range(6):
        for k in range(3):
            p = src / f"rec{g}" / f"f{k}.bin"
            p.parent.mkdir(parents=True, exist_ok=True)
            p.write_bytes(bytes([g, k]) * 100)
            rows.append(f"rec{g}/f{k}.bin,g{g},{g}")
    (tmp_path / "groups.csv").write_text("\n".join(rows) + "\n")
    coll = tmp_path / "coll"
    assert data_main(["archive", str(src), str(coll), "--groups", str(tmp_path / "groups.csv"),
                      "--pack-bytes", "4096"]) == 0
    assert data_main(["verify", str(coll), "--deep"]) == 0
    capsys.readouterr()
    assert data_main(["ls", str(coll), "--include", "rec1/*"]) == 0
    assert capsys.readouterr().out.split() == ["rec1/f0.bin", "rec1/f1.bin", "rec1/f2.bin"]
    store = LocalStore(str(coll))
    pg = PackedGroups.load(store)
    assert set(pg.groups) == {f"g{g}" for g in range(6)}
    plan = pg.plan(num_owners=2, seed=1)
    seen = set()
    for owner in range(2):
        stream = GroupStream(store, pg, plan[owner], seed=1, window=2, prefetch=1, cache=PackCache(1 << 20))
        it = iter(stream)
        first_pass = [next(it) for _ in range(stream.groups_per_pass)]
        names = {g.name for g in first_pass}
        assert len(names) == stream.groups_per_pass and not (names & seen)
        seen |= names
        g0 = first_pass[0]
        assert sorted(g0.files) == sorted(e.path for e in pg.groups[g0.name].files)
        resumed = next(iter(GroupStream(store, pg, plan[owner], seed=1, window=2, prefetch=1, start=1)))
        assert resumed.name == first_pass[1].name
    assert seen == set(pg.groups)
    assert pg.load_group(store, "g2").files["rec2/f1.bin"] == bytes([2, 1]) * 100


def test_storage_probe_local(tmp_path):
    from koochak_b200.storage.probe import probe

    rep = probe(str(tmp_path / "p"), small_count=4, large_bytes=1 << 16, streams=(1, 2), dataset_shards=2,
                shard_bytes=1 << 16, record_bytes=4096, readers=(1, 2), checkpoint_bytes=1 << 16,
                checkpoint_parts=(1, 2))
    assert rep["posix"]["exclusive_create"]["ok"] and rep["recommended_local_store"]["publish"] in ("link",
                                                                                                   "exclusive")
    assert rep["recommended_profile"]["streams"] in (1, 2)
    assert all(v["verified"] for v in rep["checkpoint"].values())
    assert os.listdir(tmp_path / "p") == []  # probe objects removed
