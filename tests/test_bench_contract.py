"""bench.py's reference arm on the CPU: the one JSON line the driver pairs
with the GPU arm's (same metric, unit, direction and workload), its
cpu_baseline and e2e objects, and the CUDA library never loaded on that
path; ranks other than 0 print nothing."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

RUN = ("import runpy, sys; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', "
       "'--warmup', '1']; runpy.run_path('bench.py', run_name='__main__'); "
       "print('VQ_LOADED', 'voyager_b200' in sys.modules)")


def _run(extra_env):
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env.update(extra_env)
    return subprocess.run([sys.executable, "-c", RUN], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=900)


def test_reference_arm_line():
    import bench

    r = _run({})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["config"]["workload"] == bench.WORKLOAD
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    # whole steps: one step of the CPU port takes about a second
    assert d["config"]["sample_rows_per_step"] == bench.ROWS
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == d["unit"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
    assert "VQ_LOADED False" in r.stdout


def test_reference_arm_other_ranks_silent():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
