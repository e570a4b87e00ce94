"""The CPU reference arm of bench.py (what the driver runs as ``--impl
reference``) prints one JSON line with the contract's keys, for the training
and the single-linear workloads."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        *args], capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def _check(d):
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_arm_training():
    d = _run("--steps", "2", "--warmup", "1", "--cpu-seq", "16")
    _check(d)
    assert d["warmup"] == 1 and "llama7b_streamed_lora" in d["config"]["workload"]


def test_reference_arm_linear():
    d = _run("--workload", "w8a8_linear_4096", "--steps", "1", "--warmup", "1",
             "--cpu-rows", "8")
    _check(d)
    assert d["unit"].startswith("TOPS")
