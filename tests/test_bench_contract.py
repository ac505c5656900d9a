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
    assert d["config"] == bench_config()  # the same workload keys as the GPU arm
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert cb["seconds"] > 0 and cb["gemvs_per_step"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def bench_config():
    sys.path.insert(0, ROOT)
    import bench

    return bench.headline_config()


def test_replayer_window_plan():
    """Windows cover exactly the K timed steps: one graph up to ONE_GRAPH
    steps, else whole cycles (at most 64 windows) plus a remainder."""
    sys.path.insert(0, ROOT)
    import bench

    class R(bench.Replayer):
        def __init__(self, n):
            self.n = n

    for n in (2, 13, 93):
        for K in (1, 3, 20, 7 * n, 2048, 2049, 20000, 100000):
            plan = R(n).plan(K)
            assert sum(p[2] for p in plan) == K
            s = 0
            for kind, first, length in plan:
                assert first == s
                if kind == "cyc":
                    assert first % n == 0 and length == plan[0][2]
                s += length
            assert len(plan) <= 65
            if K <= bench.Replayer.ONE_GRAPH:
                assert plan == [("seg", 0, K)]


@pytest.mark.gpu
def test_our_arm_line():
    steps = 52
    d = _run("--steps", str(steps), "--warmup", "3", "--no-cpu", "--no-decode", "--no-batched", "--no-orient")
    assert BASE_KEYS <= d.keys()
    assert d["steps"] == steps and d["warmup"] == 3 and d["n_gpus"] == 1 and d["higher_is_better"] is True
    assert d["config"] == bench_config()
    assert d["gpu_launches"] == steps
    assert d["warmup_steps_run"] >= 3
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
    assert w["windows"] == 8 and 0 < w["best_us"] <= w["median_us"] <= w["worst_us"]
    assert d["parity"]["ranks_ok"] == 1 and d["parity"]["max_err_over_bound"] <= 1.0
    lm = d["lmhead"]
    assert lm["parity"]["ranks_ok"] == 1 and lm["us_per_step"] > 0
    assert d["clocks"]["sm_max_mhz"] > 0
    assert d["device_status"] == 0
