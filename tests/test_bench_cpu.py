"""The CPU reference arm of bench.py (what the driver runs as ``--impl
reference``): the JSON line it prints for the training and the single-linear
workloads, and the timing of the reference's own training step it is built on
(run here on a tiny shape; the arm runs it at Llama-2-7B shapes)."""
import argparse
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

KEYS = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "cpu_baseline", "e2e")


def _check(d):
    for k in KEYS:
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_train_sample_runs_the_reference_step():
    if not os.path.exists(os.path.join(bench.REF_PKG, "lema", "__init__.py")):
        pytest.skip("the reference package is not installed in baseline/_ref")
    r = bench.reference_train_sample(2, budget_s=0.0, batch=2, seq=16, hidden=64, inter=128,
                                     vocab=256, heads=4)
    assert r["samples"] >= 1 and r["step_s_1"] > 0 and r["layer_s"] > 0
    assert abs(r["step_s_32"] - (r["step_s_1"] + 31 * r["layer_s"])) < 1e-9
    assert r["tokens_per_s_32"] == pytest.approx(2 * 16 / r["step_s_32"])


def test_reference_arm_training_line(monkeypatch):
    """The line's fields with the reference step stubbed (its own test is above):
    what was timed is reported as such, the 32-layer value under scaled_from's
    rule, and both CPU baselines are listed."""
    fake = {"tokens_per_s_32": 40.0, "step_s_32": 102.4, "step_s_1": 5.0, "layer_s": 3.14,
            "samples": 3, "timed_s": 24.4, "sample": "stub"}
    monkeypatch.setattr(bench, "reference_train_sample", lambda *a, **k: fake)
    args = argparse.Namespace(workload="llama7b_streamed_lora", steps=20, warmup=5, cpu_seq=16)
    d = bench.run_reference(args)
    _check(d)
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline_port"]["kind"] == "port"
    assert d["steps"] == 3 and d["value"] == 40.0
    assert d["ms_per_step"] == pytest.approx(24.4 / 3 * 1e3, rel=1e-3)
    assert d["scaled_from"]["timed"]["samples"] == 3
    assert d["scaled_from"]["steps_requested"] == 20


def test_reference_arm_linear():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--workload", "w8a8_linear_4096", "--steps", "1", "--warmup", "1",
                        "--cpu-rows", "8"], capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    _check(d)
    assert d["unit"].startswith("TOPS")
