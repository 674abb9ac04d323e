"""bench.py's per-workload summaries for the default line (host logic, no GPU): the child
process's JSON line is reduced to the fields the default line carries, and a failing or silent
child becomes an error entry instead of failing the whole bench."""

from __future__ import annotations

import json
import os
import subprocess
import sys
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402

LINE = {"metric": "m", "value": 2647.37, "unit": "decisions/s", "steps": 3, "warmup": 3, "ms_per_step": 385.4,
        "config": {"workload": "hybrid-2b-nvfp4-prefix-512x32q", "decisions_per_step": 1024,
                   "tokens_per_step": 79672, "path": "prefix cache"},
        "e2e": {"value": 2634.4}, "gpu_launches": 1740, "clocks": {"sm_mhz": 1477.0},
        "parity": {"max_dp": 6.3e-4, "argmax_equal": True},
        "cpu_baseline": {"value": 2.4, "cores": 16, "kind": "port", "sample": "3 requests", "_extra": 1}}


def _fake_run(rc: int, out: str, err: str = ""):
    calls = []

    def run(cmd, **kw):
        calls.append((cmd, kw))
        return types.SimpleNamespace(returncode=rc, stdout=out, stderr=err)

    return run, calls


def test_summary_of_a_child_line(monkeypatch):
    run, calls = _fake_run(0, "log line\n" + json.dumps(LINE) + "\n")
    monkeypatch.setattr(subprocess, "run", run)
    monkeypatch.setenv("WORLD_SIZE", "4")
    s = bench.other_workload("prefix", steps=3, warmup=3, cpu_sample=3)
    assert s["workload"] == "hybrid-2b-nvfp4-prefix-512x32q" and s["value"] == 2647.37 and s["e2e"] == 2634.4
    assert s["parity"]["max_dp"] == 6.3e-4 and s["cpu_baseline"] == {"value": 2.4, "cores": 16, "kind": "port",
                                                                        "sample": "3 requests"}
    cmd, kw = calls[0]
    assert cmd[2:] == ["--workload", "prefix", "--steps", "3", "--warmup", "3", "--cpu-sample", "3", "--no-extras"]
    assert "WORLD_SIZE" not in kw["env"]   # the child is a one-GPU run whatever launched the parent


def test_failing_child_is_an_error_entry(monkeypatch):
    run, _ = _fake_run(1, "", "CUDA error: out of memory")
    monkeypatch.setattr(subprocess, "run", run)
    s = bench.other_workload("ternary-batch")
    assert s["workload"] == "ternary-batch" and "exit 1" in s["error"] and "out of memory" in s["error"]


def test_silent_child_is_an_error_entry(monkeypatch):
    run, _ = _fake_run(0, "no json here\n")
    monkeypatch.setattr(subprocess, "run", run)
    assert "error" in bench.other_workload("prefix")
