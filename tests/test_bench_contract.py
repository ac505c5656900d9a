"""bench.py prints one JSON line with the keys the measurement contract names.

The reference arm (the oracle's port of the AVX2 matvec_q4k on the host cores)
runs on CPU; our arm needs a B200 and runs a short timed region.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config", "e2e", "cpu_baseline"}


def _run(*args, timeout=600):
    env = dict(os.environ, PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=timeout)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run("--impl", "reference", "--steps", "2", "--warmup", "1", "--no-decode")
    assert BASE_KEYS <= d.keys()
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    assert d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1  # warm-up is raised to at least 3
    assert d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.gpu
def test_our_arm_line():
    steps = 52
    d = _run("--steps", str(steps), "--warmup", "3", "--no-cpu", "--no-decode", "--no-batched")
    assert BASE_KEYS <= d.keys()
    assert d["steps"] == steps and d["warmup"] == 3 and d["n_gpus"] == 1 and d["higher_is_better"] is True
    assert d["gpu_launches"] == steps
    r = d["roofline"]
    assert abs(d["value"] - r["algorithmic_bytes_per_launch"] / (d["ms_per_step"] * 1e-3) / 1e9) <= 0.01 * d["value"]
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] > 0
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-3
    assert abs(r["achieved"] - d["value"]) <= 0.01 * d["value"]  # one GPU: whole-job = per-launch rate
    e = d["e2e"]
    assert e["h2d_bytes_per_step"] == 4 * d["config"]["in_dim"]
    assert e["d2h_bytes_per_step"] == 4 * d["config"]["out_dim"]
    assert 0 < e["value"] < d["value"]
    w = d["per_step_windows"]
    assert w["windows"] == steps // w["steps_per_window"] and 0 < w["best_us"] <= w["median_us"]
    assert d["clocks"]["sm_max_mhz"] > 0
    assert d["device_status"] == 0
