"""bench.py's reference arm on the CPU: the JSON line the driver reads (the metric, unit and
direction of the native arm, a cpu_baseline describing the run, an e2e object with no device
copies), and the torchrun contract that only rank 0 runs and prints."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_complete_line():
    r = run_bench({}, "--impl", "reference", "--steps", "1", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("config2")


@pytest.mark.parametrize("rank", ["1", "3"])
def test_reference_arm_runs_on_rank_zero_only(rank):
    r = run_bench({"RANK": rank, "WORLD_SIZE": "4", "LOCAL_RANK": rank}, "--impl", "reference", "--gpus", "4",
                  "--steps", "1", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
