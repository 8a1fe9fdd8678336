"""Jobs layer: torch-free imports, profiles, prepared launches, the isolated runner, artifacts."""

from __future__ import annotations

import json
import os
import signal
import subprocess
import sys
import time
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def test_jobs_import_without_torch():
    code = ("import sys\nimport koochak_b200.jobs as J\nfor n in J.__all__: getattr(J, n)\n"
            "import koochak_b200.jobs.runner, koochak_b200.jobs.isolated_exec, koochak_b200.jobs_types\n"
            "assert 'torch' not in sys.modules, 'torch imported'\n")
    subprocess.run([sys.executable, "-c", code], check=True, cwd=REPO)


def _profile(tmp_path, **extra):
    from koochak_b200.jobs import load_environment_profile

    text = {
        "version": 1, "id": "test-profile", "python": sys.executable,
        "environment": {"set": {"PATH": "/usr/bin:/bin", "PYTHONPATH": str(REPO)},
                        "create_directories": ["{run_dir}/scratch"]},
        "requirements": {"packages": {"json": "*"}},
    }
    text.update(extra)
    p = tmp_path / "profile.yaml"
    import yaml

    p.write_text(yaml.safe_dump(text))
    return load_environment_profile(p)


def test_profile_rules(tmp_path):
    from koochak_b200.jobs import EnvironmentProfile

    prof = _profile(tmp_path)
    assert prof.sha256 == _profile(tmp_path).sha256
    with pytest.raises(ValueError):
        EnvironmentProfile(profile_id="x", python=sys.executable, variables={"PATH": "/bin", "RANK": "0"})
    with pytest.raises(ValueError):
        EnvironmentProfile(profile_id="x", python=sys.executable, variables={"PATH": "bin"})
    with pytest.raises(ValueError):
        EnvironmentProfile(profile_id="x", python=sys.executable, variables={"PATH": "/bin"}, preflight=("gpu",))
    res = prof.resolve(cwd="/work", run_dir="/runs/a")
    assert res.create_directories == ("/runs/a/scratch",)


def _prepare(tmp_path, code: str, **kw):
    from koochak_b200.jobs import prepare_run, stage_run

    cfg = tmp_path / "base.yaml"
    cfg.write_text("train:\n  max_steps: 5\n  out_dir: ./x\n")
    run_dir = str(tmp_path / "run")
    prep = prepare_run(name="t1", profile=_profile(tmp_path), python_args=["-I", "-c", code, "{config}"],
                       cwd=str(tmp_path), run_dir=run_dir, base_config=cfg, **kw)
    stage_run(prep)
    return prep, run_dir


def test_prepare_stage_and_run(tmp_path):
    from koochak_b200.jobs import DeclaredOutput

    out_file = str(tmp_path / "out.txt")
    code = ("import sys, yaml\n"
            "from koochak_b200.storage.artifact import DeclaredOutput, publish_artifact\n"
            f"cfg = yaml.safe_load(open(sys.argv[1]))\nassert cfg['train']['out_dir'].endswith('run')\n"
            f"open({out_file!r}, 'w').write('hello')\n"
            f"publish_artifact(DeclaredOutput('result', {out_file!r}))\n")
    prep, run_dir = _prepare(tmp_path, code, declared_outputs=[DeclaredOutput("result", out_file)])
    manifest = json.loads(Path(prep.manifest_path).read_text())
    assert manifest["config"]["path"] == os.path.join(run_dir, "config.yaml")
    r = subprocess.run(prep.runner_argv(), capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    pre = json.loads(Path(run_dir, "preflight.json").read_text())
    assert pre["state"] == "completed" and pre["outputs"] == ["result"]
    assert Path(run_dir, "scratch").is_dir()
    # Tampering with the staged config is caught before anything runs.
    os.chmod(os.path.join(run_dir, "config.yaml"), 0o644)
    Path(run_dir, "config.yaml").write_text("train: {}\n")
    r = subprocess.run(prep.runner_argv(), capture_output=True, text=True, timeout=120)
    assert r.returncode == 78 and "config digest differs" in r.stderr


def test_preemptible_run_evacuates_with_exit_75(tmp_path):
    from koochak_b200.jobs import Preemptible

    code = ("import os, time, pathlib\n"
            "d = pathlib.Path(os.environ['KOOCHAK_EVACUATION_DIR'])\n"
            "open(os.path.join(os.path.dirname(d.as_posix()), 'started_' + d.name), 'w').close()\n"
            "for _ in range(600):\n"
            "    if (d / 'requested').exists():\n"
            "        (d / 'evacuated').touch(); raise SystemExit(1)\n"
            "    time.sleep(0.05)\n"
            "raise SystemExit(2)\n")
    prep, run_dir = _prepare(tmp_path, code, preemptible=Preemptible(grace_seconds=60, max_attempts=3))
    cfg = Path(run_dir, "config.yaml").read_text()
    assert "evacuation_enabled: true" in cfg and "resume: auto" in cfg
    proc = subprocess.Popen(prep.runner_argv(), stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
    deadline = time.time() + 60
    tmpdir = Path(os.environ.get("TMPDIR", "/tmp"))
    while time.time() < deadline and not any(p.name.startswith("started_kb-evacuation-") for p in tmpdir.iterdir()):
        time.sleep(0.05)
    proc.send_signal(signal.SIGUSR1)
    _, err = proc.communicate(timeout=60)
    assert proc.returncode == 75, err
    for p in tmpdir.iterdir():
        if p.name.startswith("started_kb-evacuation-"):
            p.unlink()


def test_artifact_manifest_roundtrip(tmp_path):
    from koochak_b200.storage.artifact import DeclaredOutput, publish_artifact, validate_artifact
    from koochak_b200.storage.immutable import write_immutable_file

    d = tmp_path / "shards"
    (d / "sub").mkdir(parents=True)
    (d / "a.bin").write_bytes(b"abc")
    (d / "sub" / "b.bin").write_bytes(b"defg")
    out = DeclaredOutput("shards", str(d), kind="directory", expected_records=2)
    m = publish_artifact(out, observed_records=2)
    assert m["size_bytes"] == 7 and [f["path"] for f in m["files"]] == ["a.bin", "sub/b.bin"]
    assert validate_artifact(out)["sha256"] == m["sha256"]
    (d / "a.bin").write_bytes(b"xyz")
    with pytest.raises(ValueError):
        validate_artifact(out)
    p = tmp_path / "imm.txt"
    assert write_immutable_file(p, b"one") is True
    assert write_immutable_file(p, b"one") is False
    with pytest.raises(FileExistsError):
        write_immutable_file(p, b"two")


def test_workflow_validation(tmp_path):
    from koochak_b200.jobs import DeclaredOutput, PreparedTask, PreparedWorkflow

    prep, _ = _prepare(tmp_path, "pass", declared_outputs=[DeclaredOutput(
        "o", str(tmp_path / "o"), provenance={"project_id": "p", "workflow_id": "w", "task_id": "a",
                                             "code_commit": "abc"})])
    t = PreparedTask("a", prep, {"gpus": 1})
    wf = PreparedWorkflow("req", "w", "p", (t,))
    spec = wf.scruffy_tasks()[0]
    assert spec["request_id"] == "req/a" and spec["argv"][:2] == [sys.executable, "-I"]
    with pytest.raises(ValueError):
        PreparedWorkflow("req", "w", "p", (PreparedTask("b", prep, {}, needs=[{"task_id": "zz",
                                                                                "condition": "succeeded"}]),))
