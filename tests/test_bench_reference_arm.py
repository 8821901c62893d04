"""bench.py --impl reference on the CPU: the JSON line the driver reads (same
metric, unit and config as the GPU arm, a cpu_baseline describing the run,
an e2e object with no host-device bytes), and the rank rule under torchrun
(rank 0 alone runs and prints; other ranks exit 0 without work). CPU only.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_arm(env_extra):
    env = dict(os.environ, **env_extra)
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    return p


def test_reference_arm_line():
    p = run_arm({})
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["metric"].startswith("MC paths/s") and d["unit"] == "paths/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] >= 3 and d["dtype"] == "f64"
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["sample"]
    e2e = d["e2e"]
    assert e2e == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    p = run_arm({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
