"""CPU: ``bench.py --impl reference`` (the oracle port on the host cores)
prints one JSON line with the benchmark contract's keys, and sizes its
per-step sample (fewer weight columns, then fewer tokens) so that ``--steps``
x the sample stays within ``--ref-budget``, down to the floor of one token
against one 128-column weight block per step."""
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def run_reference(*extra, timeout=240):
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    t0 = time.perf_counter()
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *extra],
                       capture_output=True, text=True, timeout=timeout, env=env, cwd=ROOT)
    wall = time.perf_counter() - t0
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, p.stdout
    return json.loads(lines[0]), wall


@pytest.mark.parametrize("workload", ["decode", "plumbing"])
def test_reference_arm_line_and_budget(workload):
    steps, budget = 1000, 3.0
    line, wall = run_reference("--workload", workload, "--steps", str(steps), "--warmup", "3",
                               "--ref-budget", str(budget))
    assert line["impl"] == "reference" and line["n_gpus"] == 1
    assert line["steps"] == steps and line["warmup"] == 3 and line["higher_is_better"] is True
    assert line["unit"] == "TFLOPS" and line["value"] > 0
    assert line["config"]["workload"].startswith(workload + " ")
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    assert "M=" in cpu["sample"] and "N=" in cpu["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["gpu_launches"] == 0
    # steps x per-step sample within a few budgets (the sample is sized from one
    # calibration call, so allow slack), plus interpreter start-up and data set-up
    assert line["ms_per_step"] * (steps + 3) / 1e3 < 4 * budget, line
    assert wall < 4 * budget + 60, wall


@pytest.mark.parametrize("args,env_world,why", [
    (["--warmup", "2"], "1", "--warmup must be >= 3"),
    (["--gpus", "2"], "1", "launch N>1 with torchrun"),
    (["--workload", "no_such_workload"], "1", "unknown workload"),
])
def test_contract_violations_refused(args, env_world, why):
    env = dict(os.environ, WORLD_SIZE=env_world, RANK="0", LOCAL_RANK="0")
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                       capture_output=True, text=True, timeout=120, env=env, cwd=ROOT)
    assert p.returncode == 2 and why in p.stderr, p.stderr[-500:]
    assert p.stdout.strip() == ""
