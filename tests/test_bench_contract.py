"""The bench.py contract on CPU: one JSON line on stdout with the driver's keys.

The reference arm runs on the host cores (no GPU), so its full output can be checked
here; the GPU arm's argument parsing is checked without running it.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_one_json_line():
    env = {**os.environ, "CUDA_VISIBLE_DEVICES": ""}
    # Two layers keep the CPU suite fast; the driver's run covers all 36.
    done = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "1", "--layers", "2"], capture_output=True, text=True, timeout=600, env=env,
                          cwd=ROOT)
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [line for line in done.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, done.stdout[-2000:]
    result = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in result, key
    assert result["impl"] == "reference" and result["value"] > 0 and result["steps"] == 1
    assert result["e2e"]["h2d_bytes_per_step"] == 0 and result["e2e"]["d2h_bytes_per_step"] == 0
    assert result["cpu_baseline"]["kind"] in ("port", "reference") and result["cpu_baseline"]["cores"] >= 1
    assert "workload" in result["config"]
    assert result["config"]["layers"] == 2 and result["config"]["layers_sampled"] == 2


def test_reference_arm_other_ranks_exit_quietly():
    env = {**os.environ, "CUDA_VISIBLE_DEVICES": "", "RANK": "3", "WORLD_SIZE": "4"}
    done = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "4"],
                          capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert done.returncode == 0 and not done.stdout.strip()


def test_bench_arguments():
    sys.path.insert(0, str(ROOT))
    import bench

    args = bench.parse_args([])
    assert args.gpus == 1 and args.config == 2 and args.impl == "ours" and args.only is None
    assert args.warmup >= 3
    args = bench.parse_args(["--gpus", "8", "--steps", "7", "--warmup", "4", "--only", "shadow"])
    assert (args.gpus, args.steps, args.warmup, args.only) == (8, 7, 4, "shadow")


def test_config5_topk_schedule_properties():
    """The config-5 Top-K schedule: int32 [steps, batch, k], distinct ids in [0, context)
    per row, each step keeping at least keep * k of the previous step's ids, new ids
    Zipf-concentrated near the newest token, and the same schedule for the same seed."""
    import numpy as np

    sys.path.insert(0, str(ROOT))
    import bench

    steps, batch, context, k, keep = 5, 3, 65536, 512, 0.9
    sched = bench.zipf_topk_schedule(steps, batch, context, k, keep, 1.1, seed=11)
    assert sched.shape == (steps, batch, k) and sched.dtype == np.int32
    assert ((sched >= 0) & (sched < context)).all()
    for t in range(steps):
        for b in range(batch):
            assert len(set(sched[t, b].tolist())) == k
            if t:
                shared = set(sched[t, b].tolist()) & set(sched[t - 1, b].tolist())
                assert len(shared) >= int(k * keep)
    distance = context - 1 - sched[0].astype(np.int64)
    assert np.median(distance) < context // 8  # Zipf(1.1) over distance from the newest token
    assert np.array_equal(sched, bench.zipf_topk_schedule(steps, batch, context, k, keep, 1.1, seed=11))


def test_clock_sampler_decodes_reasons(monkeypatch):
    """ClockSampler with a fake NVML: the median SM clock of the samples taken in the
    region, the max clock, and every clock-event reason bit seen (here sw_power_cap and
    hw_slowdown) by name."""
    import time
    import types

    sys.path.insert(0, str(ROOT))
    import bench

    clocks = iter([1965, 1950, 1965, 1800] + [1965] * 1000)
    bits = iter([0x4, 0x0, 0x4 | 0x8] + [0x0] * 1000)
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=0, nvmlInit=lambda: None, nvmlDeviceGetHandleByIndex=lambda index: index,
        nvmlDeviceGetMaxClockInfo=lambda handle, kind: 1965,
        nvmlDeviceGetClockInfo=lambda handle, kind: next(clocks),
        nvmlDeviceGetCurrentClocksEventReasons=lambda handle: next(bits))
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(0, period=0.001) as sampler:
        while len(sampler.samples) < 4:
            time.sleep(0.005)
    summary = sampler.summary()
    assert summary["sm_max_mhz"] == 1965 and summary["samples"] >= 4
    assert {"sw_power_cap", "hw_slowdown"} <= set(summary["reasons"])
    assert set(summary["reasons"]) <= {"sw_power_cap", "hw_slowdown"}
    # Without NVML the sampler reports no clocks instead of guessing.
    monkeypatch.setitem(sys.modules, "pynvml", None)
    with bench.ClockSampler(0) as silent:
        pass
    assert silent.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
