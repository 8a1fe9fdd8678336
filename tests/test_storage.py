import hashlib
import json
import os

import pytest
import torch

from koochak_b200.storage import checkpoint as ck
from koochak_b200.storage.store import LocalStore, StoreProfile, min_object_bytes, open_store, register_store, \
    validate_key
from koochak_b200.storage.stores_file import load_stores_file


def test_local_store_write_once(tmp_path):
    s = LocalStore(tmp_path / "s")
    info = s.put("a/b.bin", b"hello")
    assert info.size == 5 and info.sha256 == hashlib.sha256(b"hello").hexdigest()
    assert s.get("a/b.bin") == b"hello"
    assert s.get("a/b.bin", 1, 3) == b"ell"
    with pytest.raises(FileExistsError):
        s.put("a/b.bin", b"again")
    assert s.list("a/") == ["a/b.bin"]
    assert s.stat("missing") is None
    s.delete("a/b.bin")
    s.delete("a/b.bin")
    assert s.list() == []
    ex = LocalStore(tmp_path / "e", publish="exclusive")
    ex.put("k", [b"ab", b"cd"])
    assert ex.get("k") == b"abcd"
    for bad in ["", "/abs", "a//b", "a/../b", "x/.koochak-put-1"]:
        with pytest.raises(ValueError):
            validate_key(bad)


def test_open_store_and_stores_file(tmp_path, monkeypatch):
    assert isinstance(open_store(str(tmp_path)), LocalStore)
    assert open_store(f"file://{tmp_path}").root == str(tmp_path)
    f = tmp_path / "stores.yaml"
    f.write_text(f"version: 1\nstores:\n  scratch:\n    type: local\n    root: {tmp_path}/tier\n"
                 "    publish: exclusive\n    profile: {request_seconds: 0.01, stream_mb_s: 100, part_bytes: 16MiB}\n")
    specs = load_stores_file(f)
    assert specs["scratch"].profile.part_bytes == 16 * 1024 * 1024
    monkeypatch.setenv("KOOCHAK_STORES", str(f))
    st = open_store("scratch://datasets/x")
    assert st.root == f"{tmp_path}/tier/datasets/x" and st.publish == "exclusive"
    register_store("kbmem", lambda loc: LocalStore(tmp_path / "mem"))
    assert isinstance(open_store("kbmem://z"), LocalStore)
    assert min_object_bytes(StoreProfile(request_seconds=0.1, stream_mb_s=10.0)) == 3_000_000


def test_checkpoint_publish_resume_prune(tmp_path):
    store = ck.checkpoint_store(tmp_path)
    for step in (1, 2, 3, 4):
        ck.publish(store, f"step{step:09d}.pt", ck.serialize({"step": step, "next_step": step + 1, "model": {}}),
                   keep_last_k=2)
    names = sorted(os.listdir(tmp_path))
    assert "step000000004.pt" in names and "step000000002.pt" not in names
    assert os.path.islink(tmp_path / "latest.pt")
    man = (tmp_path / "step000000004.pt.ready.json").read_text()
    rec = json.loads(man)
    assert man.endswith("\n") and man == json.dumps(rec, sort_keys=True, separators=(",", ":")) + "\n"
    assert set(rec) == {"v", "artifact_id", "path", "size_bytes", "sha256", "manifest_path"}
    path, loaded = ck.resolve_auto_resume(tmp_path)
    assert loaded["step"] == 4 and path.endswith("step000000004.pt")
    # a corrupted newest checkpoint falls back to the previous valid one
    os.chmod(tmp_path / "step000000004.pt", 0o600)
    with open(tmp_path / "step000000004.pt", "ab") as fh:
        fh.write(b"x")
    assert ck.resolve_auto_resume(tmp_path)[1]["step"] == 3


def test_background_publisher_and_prefix(tmp_path):
    pub = ck.BackgroundPublisher(ck.checkpoint_store(tmp_path), keep_last_k=3)
    p = pub.submit("step000000007.pt", ck.serialize({"step": 7, "next_step": 8}), token="t")
    with pytest.raises(RuntimeError):
        pub.submit("step000000008.pt", b"x")
    path, token = pub.wait()
    assert path == p and token == "t" and ck.highest_valid_published(tmp_path) == p
    pub.close()
    m = torch.nn.Linear(2, 2)
    sd = {"module.weight": torch.zeros(2, 2), "module.bias": torch.zeros(2)}
    assert set(ck.match_state_dict_to_model(m, sd)) == {"weight", "bias"}
