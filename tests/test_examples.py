"""The shipped example files load through the public API (config template, environment profile, stores file, launch)."""

from __future__ import annotations

import os

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_config_template_has_only_known_keys():
    from koochak_b200.config import load_config, validate_unknown_keys

    cfg = load_config(os.path.join(HERE, "examples", "config_template.yaml"))
    assert validate_unknown_keys(cfg) == set()


def test_stores_example_resolves(monkeypatch):
    from koochak_b200.storage.stores_file import load_stores_file

    monkeypatch.setenv("USER", "alice")
    stores = load_stores_file(os.path.join(HERE, "examples", "storage", "stores.example.yaml"))
    assert set(stores) == {"scratch", "shared", "archive"}
    assert stores["scratch"].root == "/local/nvme/alice/koochak"
    assert stores["archive"].publish == "exclusive" and stores["archive"].verify_readback


def test_jobs_example_prepares_a_launch(monkeypatch):
    monkeypatch.chdir(HERE)
    from examples.jobs import submit

    run = submit.prepared_run()
    argv = run.runner_argv()
    assert argv[:2] == ["/opt/venv/bin/python3", "-I"]
    assert submit.prepared_run(preemptible=True).preemption is not None
