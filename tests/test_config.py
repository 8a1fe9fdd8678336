import pytest

from koochak_b200 import config as config_lib
from koochak_b200.runtime.settings import LoopSettings as _TrainSettings


def test_load_config_layering(tmp_path):
    p = tmp_path / "cfg.yaml"
    p.write_text("train:\n  max_steps: 123\n  log_every: 5\n")
    cfg = config_lib.load_config(str(p), overrides={"train": {"log_every": 9, "ckpt_every": 77}})
    assert cfg.train.max_steps == 123
    assert cfg.train.log_every == 9
    assert cfg.train.ckpt_every == 77
    assert cfg.train.eval_every == 5000
    assert cfg["optim"]["optimizer"]["name"] == "adamw"


def test_load_config_rejects_unknown_keys_and_resolves(tmp_path, monkeypatch):
    p = tmp_path / "cfg.yaml"
    p.write_text("train:\n  bogus: 1\n")
    with pytest.raises(KeyError):
        config_lib.load_config(str(p))
    monkeypatch.setenv("KB_TEST_DIR", "/tmp/x")
    p.write_text("train:\n  out_dir: ${oc.env:KB_TEST_DIR}/run\n  checkpoint_dir: ${train.out_dir}/ckpt\n")
    cfg = config_lib.load_config(str(p), overrides=["train.max_steps=7"])
    assert cfg.train.out_dir == "/tmp/x/run"
    assert cfg.train.checkpoint_dir == "/tmp/x/run/ckpt"
    assert cfg.train.max_steps == 7


def test_summarize_reports_unknown_keys(capsys):
    unknown = config_lib.summarize({"train": {"foo": 1}}, strict=False)
    assert "train.foo" in unknown
    assert "unknown keys" in capsys.readouterr().out
    with pytest.raises(ValueError):
        config_lib.summarize({"train": {"foo": 1}}, strict=True)


def test_get_section_required_behavior():
    cfg = {"train": {"max_steps": 1}}
    assert config_lib.get_section(cfg, "train") is not None
    assert config_lib.get_section(cfg, "data", required=False) is None
    with pytest.raises(KeyError):
        config_lib.get_section(cfg, "data")


def test_ddp_options_known_and_exclusive():
    cfg = {"train": {"ddp": True, "ddp_static_graph": True, "ddp_bucket_cap_mb_list": [1, 16],
                     "ddp_broadcast_buffers": False}}
    assert not config_lib.summarize(cfg, strict=False)
    s = _TrainSettings.from_cfg(cfg["train"])
    assert s.ddp_enabled and s.ddp_static_graph and s.ddp_bucket_cap_mb_list == (1, 16)
    assert s.ddp_broadcast_buffers is False
    with pytest.raises(ValueError, match="only one"):
        _TrainSettings.from_cfg({"ddp_bucket_cap_mb": 16, "ddp_bucket_cap_mb_list": [1, 16]})
