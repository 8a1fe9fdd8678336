"""GPU-health rules, verdict timing, node queries and Slurm actions, on CPU with fake readings.

Behaviours follow the reference's health tests (koochak tests/test_gpu_health.py):
two consecutive non-thermal faults fail, a good reading resets the streak, a
thermal episode fails only after two hours of continuous evidence, the power
brake stays fast during a thermal episode, Slurm requeue / cancel / exit run
exactly their commands (and none from nested steps or when disabled). No GPU
and no scheduler are touched: time and command execution are injected.
"""

from __future__ import annotations

import json
import subprocess
from pathlib import Path

import pytest
import torch

from koochak_b200.health import gpu as gh
from koochak_b200.health.gpu import (PRIMARY_QUERY_FIELDS, THERMAL_GRACE_SECONDS, THERMAL_MAX_SAMPLE_GAP_SECONDS,
                                     GpuHealthSample, GpuHealthWatchdog, evaluate_sample, parse_nvidia_smi_csv)
from koochak_b200.health.node_query import query_node_samples


def _sample(**kw) -> GpuHealthSample:
    base = dict(step=20, rank=0, local_rank=0, world_size=1, hostname="node-3", slurm_node="node-3", cuda_device=2,
                gpu_query_id="2", gpu_index="2", gpu_uuid="GPU-11111111-2222-3333-4444-555555555555",
                gpu_name="NVIDIA B200", gpu_temp_c=88.0, memory_temp_c=90.0, pstate="P0", power_draw_w=600.0,
                power_limit_w=1000.0, sm_clock_mhz=600.0, mem_clock_mhz=3996.0, max_sm_clock_mhz=1965.0,
                gpu_util_pct=100.0, mem_util_pct=40.0, throttle_active_mask="0x20", sw_thermal_slowdown=True,
                hw_slowdown=False, hw_thermal_slowdown=False, hw_power_brake_slowdown=False, sw_power_cap=False,
                timestamp_unix=1.0)
    base.update(kw)
    return GpuHealthSample(**base)


HEALTHY = dict(gpu_temp_c=55.0, memory_temp_c=60.0, sm_clock_mhz=1900.0, sw_thermal_slowdown=False)


def test_rules_name_every_reason_in_order():
    assert evaluate_sample(_sample()) == ["sw_thermal_slowdown", "gpu_temp_high", "sm_clock_low"]
    assert evaluate_sample(_sample(**HEALTHY)) == []
    assert evaluate_sample(_sample(**HEALTHY, sw_power_cap=True)) == []  # a power-capped B200 is normal
    assert evaluate_sample(_sample(gpu_util_pct=40.0)) == []  # idle GPUs are not judged
    assert evaluate_sample(_sample(gpu_util_pct=None)) == []
    assert evaluate_sample(_sample(**{**HEALTHY, "memory_temp_c": 94.0})) == ["memory_temp_high"]


def test_parse_row_keeps_identity(monkeypatch):
    monkeypatch.setenv("LOCAL_RANK", "3")
    values = {"index": "5", "uuid": "GPU-abc", "name": "NVIDIA B200", "temperature.gpu": "70", "clocks.sm": "1900",
              "clocks.max.sm": "1965", "utilization.gpu": "97", "clocks_throttle_reasons.hw_slowdown": "Active",
              "power.draw": "812.5 W"}
    row = ",".join(values.get(f, "N/A") for f in PRIMARY_QUERY_FIELDS)
    s = parse_nvidia_smi_csv(stdout=row + "\n", fields=PRIMARY_QUERY_FIELDS, step=40, rank=7, world_size=8,
                             hostname="h", slurm_node="n", cuda_device=5, gpu_query_id="5")
    assert (s.rank, s.local_rank, s.slurm_node, s.gpu_uuid, s.gpu_index) == (7, 3, "n", "GPU-abc", "5")
    assert s.hw_slowdown and not s.sw_power_cap and s.memory_temp_c is None and s.power_draw_w == 812.5
    assert parse_nvidia_smi_csv(stdout="", fields=PRIMARY_QUERY_FIELDS, step=0, rank=0, world_size=1, hostname="h",
                                slurm_node="n", cuda_device=0, gpu_query_id="0") is None


@pytest.fixture
def watch(tmp_path):
    clock = [0.0]
    w = GpuHealthWatchdog(device=torch.device("cuda", 0), out_dir=str(tmp_path), rank=0, world_size=1,
                          clock=lambda: clock[0])

    def at(seconds, sample):
        clock[0] = seconds
        w.read_sample = lambda step: sample
        return w.check_local(20)

    return at


def test_two_consecutive_faults_fail_and_good_reading_resets(watch):
    bad = _sample(**HEALTHY, hw_power_brake_slowdown=True)
    assert watch(0, bad) is None
    assert watch(30, _sample(**HEALTHY)) is None  # reset
    assert watch(60, bad) is None
    failure = watch(90, bad)
    assert failure is not None and failure.reasons == ["hw_power_brake_slowdown"] and failure.consecutive_failures == 2


@pytest.mark.parametrize("overrides", [{}, {"gpu_temp_c": 70.0, "sm_clock_mhz": 1900.0},
                                       {"sw_thermal_slowdown": False},
                                       {"gpu_temp_c": 50.0, "sw_thermal_slowdown": False, "memory_temp_c": 96.0},
                                       {"hw_thermal_slowdown": True, "hw_slowdown": True}])
def test_heat_fails_only_after_two_hours(watch, tmp_path, overrides):
    s = _sample(**overrides)
    for t in range(0, THERMAL_GRACE_SECONDS, 30):
        assert watch(t, s) is None
    assert watch(THERMAL_GRACE_SECONDS - 0.001, s) is None
    failure = watch(THERMAL_GRACE_SECONDS, s)
    assert failure is not None and failure.thermal_duration_seconds == THERMAL_GRACE_SECONDS
    assert failure.consecutive_failures == THERMAL_GRACE_SECONDS // 30 + 2
    rows = (tmp_path / "gpu_health" / "gpu_health_rank0.jsonl").read_text().splitlines()
    assert json.loads(rows[-1])["thermal_grace_seconds"] == THERMAL_GRACE_SECONDS
    assert json.loads(rows[-2])["thermal_duration_seconds"] < THERMAL_GRACE_SECONDS


@pytest.mark.parametrize("break_kind", ["healthy", "missing", "idle", "gap"])
def test_heat_episode_restarts_without_continuous_evidence(watch, break_kind):
    for t in range(0, THERMAL_GRACE_SECONDS, 30):
        assert watch(t, _sample()) is None
    now = THERMAL_GRACE_SECONDS
    if break_kind == "gap":
        now += THERMAL_MAX_SAMPLE_GAP_SECONDS + 1
        assert watch(now, _sample()) is None
    else:
        other = {"healthy": _sample(**HEALTHY), "idle": _sample(gpu_util_pct=0.0), "missing": None}[break_kind]
        assert watch(now, other) is None
    assert watch(now + 30, _sample()) is None


@pytest.mark.parametrize("fault", ["hw_power_brake_slowdown", "hw_slowdown", "sm_clock_low"])
def test_fault_streak_does_not_count_thermal_samples(watch, fault):
    assert watch(0, _sample()) is None
    kw = dict(HEALTHY)
    if fault == "sm_clock_low":
        kw["sm_clock_mhz"] = 500.0
    else:
        kw[fault] = True
    assert watch(30, _sample(**kw)) is None
    failure = watch(60, _sample(**kw))
    assert failure is not None and failure.reasons == [fault] and failure.consecutive_failures == 2


def test_power_brake_stays_fast_while_hot(watch):
    s = _sample(hw_power_brake_slowdown=True, hw_slowdown=True)
    assert watch(0, s) is None
    failure = watch(30, s)
    assert failure is not None and failure.reasons == ["hw_power_brake_slowdown"]


def test_wall_clock_jump_does_not_end_grace(watch):
    assert watch(0, _sample(timestamp_unix=0.0)) is None
    assert watch(30, _sample(timestamp_unix=1e6)) is None


class _Recorder:
    def __init__(self, pending="8101 8102"):
        self.cmds = []
        self.pending = pending

    def __call__(self, cmd):
        self.cmds.append(list(cmd))
        out = self.pending if cmd[0] == "squeue" else ""
        return {"cmd": " ".join(cmd), "returncode": 0, "stdout": out, "stderr": ""}


def _watchdog(tmp_path, runner):
    return GpuHealthWatchdog(device=torch.device("cuda", 0), out_dir=str(tmp_path), rank=0, world_size=1,
                             runner=runner)


FAIL = [{"slurm_node": "node-3", "hostname": "node-3.cluster", "reasons": ["hw_slowdown"]}]


@pytest.fixture
def slurm_env(monkeypatch):
    for k in ("SCRUFFY_JOB_ID", "SCRUFFY_ROOT", "SLURM_STEP_ID", "SLURM_STEPID", "SLURM_JOB_NODELIST",
              "KOOCHAK_GPU_HEALTH_SLURM_DISABLE", "KOOCHAK_GPU_HEALTH_SLURM_ACTION"):
        monkeypatch.delenv(k, raising=False)
    monkeypatch.setenv("SLURM_JOB_ID", "7000")
    monkeypatch.setenv("SLURM_JOB_NAME", "train")
    monkeypatch.setenv("USER", "me")
    return monkeypatch


def test_slurm_default_is_exit(slurm_env, tmp_path):
    rec = _Recorder()
    w = _watchdog(tmp_path, rec)
    assert w.slurm_action == "exit" and w.perform_slurm_recovery(FAIL) == [] and rec.cmds == []


def test_slurm_requeue_excludes_bad_nodes_everywhere(slurm_env, tmp_path):
    slurm_env.setenv("KOOCHAK_GPU_HEALTH_SLURM_ACTION", "requeue")
    rec = _Recorder()
    w = _watchdog(tmp_path, rec)
    w.perform_slurm_recovery(FAIL)
    assert rec.cmds == [["scontrol", "update", "JobId=7000", "ExcNodeList=node-3"],
                        ["squeue", "-h", "-u", "me", "-t", "PENDING", "-n", "train", "-o", "%i"],
                        ["scontrol", "update", "JobId=8101", "ExcNodeList=node-3"],
                        ["scontrol", "update", "JobId=8102", "ExcNodeList=node-3"],
                        ["scontrol", "requeue", "7000"]]


def test_slurm_cancel_uses_scancel(slurm_env, tmp_path):
    slurm_env.setenv("KOOCHAK_GPU_HEALTH_SLURM_ACTION", "cancel")
    rec = _Recorder(pending="")
    _watchdog(tmp_path, rec).perform_slurm_recovery(FAIL)
    assert [c[0] for c in rec.cmds] == ["squeue", "scancel"] and ["scontrol", "requeue", "7000"] not in rec.cmds


@pytest.mark.parametrize("env", [{"SLURM_STEP_ID": "3"}, {"SCRUFFY_JOB_ID": "x"},
                                 {"KOOCHAK_GPU_HEALTH_SLURM_DISABLE": "1"}])
def test_slurm_never_touched_from_nested_or_disabled(slurm_env, tmp_path, env):
    slurm_env.setenv("KOOCHAK_GPU_HEALTH_SLURM_ACTION", "requeue")
    for k, v in env.items():
        slurm_env.setenv(k, v)
    rec = _Recorder()
    w = _watchdog(tmp_path, rec)
    assert w.perform_slurm_recovery(FAIL) == [] and rec.cmds == []
    if "KOOCHAK_GPU_HEALTH_SLURM_DISABLE" not in env:
        assert w.slurm_action == "exit" and w.slurm_mutation_blocked_reason


def test_bad_nodes_follow_the_job_nodelist(slurm_env, tmp_path):
    slurm_env.setenv("SLURM_JOB_NODELIST", "node-[1-4]")

    def runner(cmd):
        return {"returncode": 0, "stdout": "node-1\nnode-3\n", "stderr": "", "cmd": " ".join(cmd)}

    assert _watchdog(tmp_path, runner).bad_nodes_from_failures(
        [{"slurm_node": "unknown", "hostname": "node-3.cluster"}]) == ["node-3"]


def test_failure_summary_file(slurm_env, tmp_path):
    w = _watchdog(tmp_path, _Recorder())
    path = Path(w.write_failure_summary(step=40, failures=FAIL, checkpoint_path="/x/step000000040.pt"))
    assert path.name == "gpu_health_failure_step000000040.json"
    data = json.loads(path.read_text())
    assert data["bad_nodes"] == ["node-3"] and data["slurm_action"] == "exit" and data["step"] == 40


def _rows(ids, uuids, **over):
    out = []
    for i, u in zip(ids, uuids):
        v = {"index": i, "uuid": u, "name": "B200", "temperature.gpu": "60", "clocks.sm": "1900",
             "clocks.max.sm": "1965", "utilization.gpu": "99"}
        v.update(over)
        out.append(",".join(v.get(f, "N/A") for f in PRIMARY_QUERY_FIELDS))
    return "\n".join(out)


def _node(tmp_path, ids):
    ws = []
    for r, qid in enumerate(ids):
        w = GpuHealthWatchdog(device=torch.device("cuda", r), out_dir=str(tmp_path), rank=r, world_size=len(ids))
        w.gpu_query_id = qid
        w.nvidia_smi = "nvidia-smi"
        ws.append(w)
    return ws


def test_node_query_matches_rows_by_index_or_uuid(tmp_path):
    ws = _node(tmp_path, ["GPU-bbb", "0"])
    seen = []

    def run(argv):
        seen.append(argv)
        return subprocess.CompletedProcess(argv, 0, _rows(["0", "1"], ["GPU-aaa", "GPU-bbbb-1"]), "")

    samples = query_node_samples(ws, 12, run=run)
    assert [s.gpu_uuid for s in samples] == ["GPU-bbbb-1", "GPU-aaa"] and [s.rank for s in samples] == [0, 1]
    assert seen[0][:3] == ["nvidia-smi", "-i", "GPU-bbb,0"]


@pytest.mark.parametrize("case", ["dup", "short", "missing_temp", "negative"])
def test_node_query_refuses_untrustworthy_rows(tmp_path, case):
    ws = _node(tmp_path, ["0", "1"])
    stdout = {"dup": _rows(["0", "1"], ["GPU-a", "GPU-a"]), "short": _rows(["0"], ["GPU-a"]),
              "missing_temp": _rows(["0", "1"], ["GPU-a", "GPU-b"], **{"temperature.gpu": "N/A"}),
              "negative": _rows(["0", "1"], ["GPU-a", "GPU-b"], **{"power.draw": "-5"})}[case]
    with pytest.raises(RuntimeError):
        query_node_samples(ws, 0, run=lambda argv: subprocess.CompletedProcess(argv, 0, stdout, ""))


def test_node_query_falls_back_to_older_field_list(tmp_path):
    ws = _node(tmp_path, ["0"])
    calls = []

    def run(argv):
        calls.append(argv)
        if len(calls) == 1:
            return subprocess.CompletedProcess(argv, 2, "", "Field temperature.memory is not a valid field")
        fields = gh.FALLBACK_QUERY_FIELDS
        v = {"index": "0", "uuid": "GPU-a", "temperature.gpu": "60", "clocks.sm": "1900", "utilization.gpu": "99"}
        return subprocess.CompletedProcess(argv, 0, ",".join(v.get(f, "N/A") for f in fields), "")

    (s,) = query_node_samples(ws, 0, run=run)
    assert len(calls) == 2 and s.memory_temp_c is None and s.gpu_uuid == "GPU-a"
