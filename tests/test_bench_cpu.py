"""The CPU side of bench.py: the reference arm's JSON line (the timed oracle
port on one pinned core) and its contract keys, its rank handling under a
multi-rank launch, and the row extrapolation both CPU figures use."""
import importlib.util
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_extrapolation_is_a_fixed_part_plus_a_part_linear_in_rows(bench):
    fixed, per_row = 0.5, 0.01
    t = lambda rows: fixed + per_row * rows  # noqa: E731
    got = bench._extrapolate(t(16), t(64), 16, 64)
    assert abs(got - (fixed + per_row * bench.GLOBAL_BATCH)) < 1e-9
    # a fixed part estimated below zero is clamped to zero, never subtracted
    per_row = (0.5 - 0.1) / 48
    assert abs(bench._extrapolate(0.1, 0.5, 16, 64) - per_row * bench.GLOBAL_BATCH) < 1e-9


def _run(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                          env=e, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line(bench):
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "steps/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["warmup"] >= 3 and line["steps"] == 1
    assert line["config"]["workload"] == bench.WORKLOAD
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] == 1 and cb["value"] == line["value"]
    assert "1 pinned host core" in cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "steps/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"],
             env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0 and r.stdout.strip() == ""
