"""Measure the storage semantics and performance the stores rely on.

(reference: koochak/storage/probe.py:644-889)

    python -m koochak_b200.storage.probe /path/on/a/filesystem [--json]
    python -m koochak_b200.storage.probe scheme://bucket/prefix --checkpoint-bytes 4GiB

For a local path (FUSE mounts included) it first checks POSIX behaviour:
exclusive create, rename-over, hard links, symlinks, fsync, whether an
unclosed file is visible, and how long a closed file takes to read back with
its exact bytes. From those it recommends ``LocalStore`` settings
(``publish="link"`` when hard links work, else ``"exclusive"``;
``verify_readback`` and ``read_settle_seconds`` when read-after-close lags),
then exercises the store API: the contract (put/get/ranged get/stat/list
agree, create-only puts, delete), small-object put/get/stat latency,
listing, and large-object throughput -- one stream, ranged parallel reads of
one object, many objects at once, each cold (page cache dropped where the
filesystem allows) and warm -- from which it recommends a ``StoreProfile``. Optional phases: a checkpoint-sized payload written as 1..N
concurrent parts and timed until every part reads back with its exact
SHA-256; and a synthetic ``ShardWriter`` dataset read back with
``assign_shards``. Everything lives under a fresh ``koochak-probe-<id>``
prefix that is removed afterwards unless ``keep=True``.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import platform
import shutil
import sys
import tempfile
import time
import uuid
from concurrent.futures import ThreadPoolExecutor
from typing import Any, Callable, Dict, List, Optional, Sequence

from ..utils.sizes import parse_size
from .store import LocalStore, Store, open_store

__all__ = ["probe", "main"]

_MB = 1_000_000


def _pct(xs: Sequence[float]) -> Dict[str, float]:
    s = sorted(xs)
    if not s:
        return {}
    pick = lambda q: s[min(len(s) - 1, int(q * (len(s) - 1) + 0.5))]  # noqa: E731
    return {"p50_ms": pick(0.5) * 1e3, "p90_ms": pick(0.9) * 1e3, "max_ms": s[-1] * 1e3}


def _timed(fn: Callable[[], Any]) -> float:
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


def _check(out: Dict[str, Any], name: str, fn: Callable[[], Optional[Dict[str, Any]]]) -> None:
    try:
        extra = fn() or {}
        out[name] = {"ok": True, **extra}
    except OSError as exc:
        out[name] = {"ok": False, "error": f"{type(exc).__name__}: {exc.strerror or exc}"}
    except AssertionError as exc:
        out[name] = {"ok": False, "error": str(exc)}


def _posix(d: str, small: bytes, large: bytes, settle_timeout: float) -> Dict[str, Any]:
    res: Dict[str, Any] = {}
    p = lambda n: os.path.join(d, n)  # noqa: E731

    def excl():
        with open(p("x"), "xb") as f:
            f.write(small)
        try:
            open(p("x"), "xb").close()
        except FileExistsError:
            return None
        raise AssertionError("O_EXCL create succeeded on an existing file")

    def rename():
        for n, b in (("r1", b"1"), ("r2", b"2")):
            with open(p(n), "wb") as f:
                f.write(b)
        os.replace(p("r1"), p("r2"))
        assert open(p("r2"), "rb").read() == b"1", "rename-over did not replace the target"

    def link():
        with open(p("l1"), "wb") as f:
            f.write(small)
        os.link(p("l1"), p("l2"))
        try:
            os.link(p("l1"), p("l2"))
        except FileExistsError:
            return None
        raise AssertionError("link over an existing name succeeded")

    def symlink():
        os.symlink("x", p("s"))

    def fsync():
        fd = os.open(p("f"), os.O_CREAT | os.O_WRONLY, 0o644)
        try:
            os.write(fd, small)
            return {"seconds": _timed(lambda: os.fsync(fd))}
        finally:
            os.close(fd)

    def unclosed():
        f = open(p("u"), "wb")
        try:
            f.write(small)
            f.flush()
            seen = os.path.exists(p("u"))
            return {"visible_before_close": seen}
        finally:
            f.close()

    def readback():
        with open(p("big"), "wb") as f:
            f.write(large)
        t0 = time.perf_counter()
        while True:
            with open(p("big"), "rb") as f:
                if f.read() == large:
                    return {"settle_seconds": time.perf_counter() - t0}
            if time.perf_counter() - t0 > settle_timeout:
                raise AssertionError(f"closed file did not read back within {settle_timeout}s")
            time.sleep(0.05)

    for name, fn in (("exclusive_create", excl), ("rename_over", rename), ("hard_link", link),
                     ("symlink", symlink), ("fsync", fsync), ("unclosed_file", unclosed), ("readback", readback)):
        _check(res, name, fn)
    return res


def _recommend_local(posix: Dict[str, Any]) -> Dict[str, Any]:
    rb = posix.get("readback", {})
    settle = float(rb.get("settle_seconds", 0.0)) if rb.get("ok") else None
    rec: Dict[str, Any] = {"publish": "link" if posix.get("hard_link", {}).get("ok") else "exclusive",
                           "fsync": bool(posix.get("fsync", {}).get("ok"))}
    if settle is None or settle > 0.01:
        rec["verify_readback"] = True
        rec["read_settle_seconds"] = max(5.0, 4 * (settle or 15.0))
    return rec


def _semantics(store: Store, prefix: str, small: bytes) -> Dict[str, Any]:
    """The store contract the checkpoint and dataset code relies on, checked on one small object."""

    key = f"{prefix}/semantics"
    info = store.put(key, small)
    seen = store.stat(key)
    out: Dict[str, Any] = {
        "put_info_matches": info.size == len(small),
        "get_matches": store.get(key) == small,
        "range_get_matches": store.get(key, 1, 3) == small[1:4],
        "stat_size_matches": seen is not None and seen.size == len(small),
        "listed_after_put": key in store.list(f"{prefix}/"),
    }
    try:
        store.put(key, small)
        out["create_only"] = False
    except FileExistsError:
        out["create_only"] = True
    store.delete(key)
    out["absent_after_delete"] = store.stat(key) is None
    out["ok"] = all(out.values())
    return out


def _evict(store: Store, key: str) -> bool:
    """Best effort: drop a local file's cached pages, so the next read of it comes from the device."""

    path = store.local_path(key)
    fadvise = getattr(os, "posix_fadvise", None)
    if path is None or fadvise is None:
        return False
    fd = os.open(path, os.O_RDONLY)
    try:
        fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
        return True
    except OSError:
        return False
    finally:
        os.close(fd)


def _tagged(data: bytes, tag: int) -> bytes:
    """``data`` with a distinct 16-byte head, so separate objects never share cached pages by content."""

    return tag.to_bytes(16, "little") + data[16:]


def _store_phase(store: Store, prefix: str, small: bytes, count: int, large: bytes,
                 streams: Sequence[int]) -> Dict[str, Any]:
    out: Dict[str, Any] = {"semantics": _semantics(store, prefix, small)}
    keys = [f"{prefix}/small/{i:05d}" for i in range(count)]
    out["small_put"] = _pct([_timed(lambda k=k: store.put(k, small)) for k in keys])
    out["small_stat"] = _pct([_timed(lambda k=k: store.stat(k)) for k in keys])
    out["small_get"] = _pct([_timed(lambda k=k: store.get(k)) for k in keys])
    listed: List[str] = []
    out["list_seconds"] = _timed(lambda: listed.extend(store.list(f"{prefix}/small/")))
    out["list_complete"] = sorted(listed) == keys

    # Large objects: a separate object for every cold measurement (reading warms what it touches).
    n_max, size = max(streams), len(large)
    single, ranged = f"{prefix}/large/single", f"{prefix}/large/ranged"
    many = [f"{prefix}/large/{j:03d}" for j in range(n_max)]
    put_one = _timed(lambda: store.put(single, _tagged(large, 0)))
    with ThreadPoolExecutor(max_workers=n_max + 1) as pool:
        put_all = _timed(lambda: list(pool.map(lambda jk: store.put(jk[1], _tagged(large, jk[0] + 1)),
                                               enumerate([ranged, *many]))))
    cold_ok = all([_evict(store, k) for k in (single, ranged, *many)])
    cold = _timed(lambda: store.get(single))
    warm = _timed(lambda: store.get(single))
    out["large_single_stream"] = {"bytes": size, "put_mb_s": size / put_one / _MB, "cold_get_mb_s": size / cold / _MB,
                                  "warm_get_mb_s": size / warm / _MB, "cold_is_cold": cold_ok}
    part = -(-size // n_max)

    def ranged_read() -> None:
        with ThreadPoolExecutor(max_workers=n_max) as pool:
            got = sum(pool.map(lambda off: len(store.get(ranged, off, min(part, size - off))), range(0, size, part)))
        if got != size:
            raise RuntimeError(f"ranged read returned {got} of {size} bytes")

    cold = _timed(ranged_read)
    warm = _timed(ranged_read)
    out["large_ranged"] = {"ranges": n_max, "part_bytes": part, "cold_get_mb_s": size / cold / _MB,
                           "warm_get_mb_s": size / warm / _MB}
    conc: Dict[str, Any] = {"put_streams": n_max + 1, "put_mb_s": size * (n_max + 1) / put_all / _MB}
    with ThreadPoolExecutor(max_workers=n_max) as pool:
        t = _timed(lambda: list(pool.map(store.get, many)))
    conc[f"cold_get_{n_max}_streams_mb_s"] = size * n_max / t / _MB
    for n in streams:
        with ThreadPoolExecutor(max_workers=n) as pool:
            t = _timed(lambda: list(pool.map(store.get, many[:n])))
        conc[f"warm_get_{n}_streams_mb_s"] = size * n / t / _MB
        out[f"read_{n}_streams_mb_s"] = conc[f"warm_get_{n}_streams_mb_s"]
    out["large_concurrent"] = conc
    for k in (*keys, single, ranged, *many):
        store.delete(k)
    return out


def _recommend_profile(r: Dict[str, Any], streams: Sequence[int]) -> Dict[str, Any]:
    one = r.get("large_single_stream", {}).get("cold_get_mb_s") or r.get(f"read_{streams[0]}_streams_mb_s", 100.0)
    best_n = max(streams, key=lambda n: r.get(f"read_{n}_streams_mb_s", 0.0))
    ranged = r.get("large_ranged", {})
    range_streams = ranged.get("ranges", 1) if ranged.get("cold_get_mb_s", 0.0) > 1.5 * one else 1
    req = r.get("small_get", {}).get("p50_ms", 1.0) / 1e3
    return {"request_seconds": max(req, 1e-4), "stream_mb_s": one, "streams": int(best_n),
            "range_streams": int(range_streams), "part_bytes": 64 * 1024 * 1024,
            "list_is_cheap": r.get("list_seconds", 1.0) < 0.5}


def _checkpoint_phase(store: Store, prefix: str, total: int, parts: Sequence[int], settle: float) -> Dict[str, Any]:
    out: Dict[str, Any] = {}
    for n in parts:
        size = total // n
        blobs = [os.urandom(min(size, 1 << 20)) * (size // min(size, 1 << 20)) for _ in range(n)]
        keys = [f"{prefix}/ckpt-{n}-{j}" for j in range(n)]
        digests = [hashlib.sha256(b).hexdigest() for b in blobs]
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=n) as pool:
            list(pool.map(lambda kb: store.put(kb[0], kb[1]), zip(keys, blobs)))
            wrote = time.perf_counter() - t0
            while True:
                ok = all(hashlib.sha256(d).hexdigest() == g for d, g in zip(pool.map(store.get, keys), digests))
                if ok or time.perf_counter() - t0 > settle + wrote:
                    break
                time.sleep(0.1)
        out[f"{n}_parts"] = {"write_mb_s": sum(map(len, blobs)) / wrote / _MB,
                             "visible_seconds": time.perf_counter() - t0, "verified": ok}
    return out


def _dataset_phase(store: Store, prefix: str, shards: int, shard_bytes: int, record_bytes: int,
                   readers: Sequence[int]) -> Dict[str, Any]:
    from ..data.shards import TAR, ShardWriter, assign_shards, read_shard

    rec = os.urandom(record_bytes)
    t0 = time.perf_counter()
    with ShardWriter(store, f"{prefix}/dataset", target_bytes=shard_bytes) as w:
        per = max(1, shard_bytes // (record_bytes + 1024))
        for i in range(shards * per):
            w.add({"__key__": f"r{i:08d}", "bin": rec})
    idx = w.index
    out: Dict[str, Any] = {"build_mb_s": idx.size_bytes / (time.perf_counter() - t0) / _MB}
    for n in readers:
        def work(k: int) -> int:
            return sum(sum(1 for _ in TAR.decode(read_shard(store, s)))
                       for s in assign_shards(idx, worker=k, num_workers=n))
        t = time.perf_counter()
        with ThreadPoolExecutor(max_workers=n) as pool:
            assert sum(pool.map(work, range(n))) == idx.records
        out[f"read_{n}_readers_mb_s"] = idx.size_bytes / (time.perf_counter() - t) / _MB
    return out


def probe(location: str, *, small_count: int = 64, small_bytes: int = 4096, large_bytes: int = 64 << 20,
          streams: Sequence[int] = (1, 8), settle_timeout: float = 60.0, checkpoint_bytes: int = 0,
          checkpoint_parts: Sequence[int] = (1, 4), dataset_shards: int = 0, shard_bytes: int = 64 << 20,
          record_bytes: int = 1 << 20, readers: Sequence[int] = (1, 4), keep: bool = False,
          stores_file: Optional[str] = None) -> Dict[str, Any]:
    for what, v, lo in (("small_count", small_count, 4), ("small_bytes", small_bytes, 4),
                        ("large_bytes", large_bytes, 64)):
        if type(v) is not int or v < lo:
            raise ValueError(f"{what} must be an integer >= {lo}")
    if not streams or any(type(n) is not int or n < 1 for n in streams):
        raise ValueError("streams must be positive integers")
    run_id = f"koochak-probe-{uuid.uuid4().hex[:12]}"
    small, large = os.urandom(small_bytes), os.urandom(large_bytes)
    report: Dict[str, Any] = {"location": str(location), "run_id": run_id, "host": platform.node(),
                              "python": platform.python_version()}
    t0 = time.perf_counter()
    local_dir = None if "://" in str(location) else os.path.abspath(str(location))
    if local_dir is not None:
        os.makedirs(local_dir, exist_ok=True)
        scratch = tempfile.mkdtemp(prefix=run_id + "-posix-", dir=local_dir)
        try:
            report["posix"] = _posix(scratch, small, large, settle_timeout)
        finally:
            shutil.rmtree(scratch, ignore_errors=True)
        report["recommended_local_store"] = _recommend_local(report["posix"])
        kw = {k: v for k, v in report["recommended_local_store"].items()
              if k in ("publish", "fsync", "verify_readback", "read_settle_seconds")}
        store: Store = LocalStore(local_dir, **kw)
    else:
        store = open_store(location, stores_file=stores_file)
    try:
        report["store"] = _store_phase(store, run_id, small, small_count, large, tuple(streams))
        report["recommended_profile"] = _recommend_profile(report["store"], tuple(streams))
        if checkpoint_bytes:
            report["checkpoint"] = _checkpoint_phase(store, run_id, checkpoint_bytes, checkpoint_parts,
                                                     settle_timeout)
        if dataset_shards:
            report["dataset"] = _dataset_phase(store, run_id, dataset_shards, shard_bytes, record_bytes, readers)
    finally:
        if not keep:
            for k in store.list(run_id):
                try:
                    store.delete(k)
                except OSError:
                    pass
            if local_dir is not None:
                shutil.rmtree(os.path.join(local_dir, run_id), ignore_errors=True)
    report["seconds"] = time.perf_counter() - t0
    return report


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m koochak_b200.storage.probe", description=__doc__.split("\n\n")[0])
    ap.add_argument("location")
    ap.add_argument("--json", action="store_true", help="print the full JSON report")
    ap.add_argument("--small-count", type=int, default=64)
    ap.add_argument("--large-bytes", type=parse_size, default=64 << 20)
    ap.add_argument("--streams", default="1,8")
    ap.add_argument("--settle-timeout", type=float, default=60.0)
    ap.add_argument("--checkpoint-bytes", type=parse_size, default=0)
    ap.add_argument("--dataset-shards", type=int, default=0)
    ap.add_argument("--keep", action="store_true")
    ap.add_argument("--stores", default=None)
    a = ap.parse_args(argv)
    rep = probe(a.location, small_count=a.small_count, large_bytes=a.large_bytes,
                streams=tuple(int(x) for x in a.streams.split(",")), settle_timeout=a.settle_timeout,
                checkpoint_bytes=a.checkpoint_bytes, dataset_shards=a.dataset_shards, keep=a.keep,
                stores_file=a.stores)
    if a.json:
        print(json.dumps(rep, indent=2, sort_keys=True, default=str))
    else:
        for k in ("recommended_local_store", "recommended_profile"):
            if k in rep:
                print(f"{k}: {json.dumps(rep[k], sort_keys=True)}")
        st = rep.get("store", {})
        print(f"small get p50 {st.get('small_get', {}).get('p50_ms', 0):.2f} ms; "
              + "; ".join(f"{k} {v:.0f}" for k, v in st.items() if k.endswith("mb_s")))
    return 0


if __name__ == "__main__":
    sys.exit(main())
