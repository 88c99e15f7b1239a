"""bench.py's reference arm on the CPU: reef's own engine (oracle/_ref) timed
on a bounded sample of config 3, printing the one JSON line the driver reads,
with the same metric as the GPU arm; ranks other than 0 print nothing."""
import json
import os
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run(env_extra: dict, *args: str) -> subprocess.CompletedProcess:
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_the_contract_line():
    p = run({}, "--impl", "reference", "--steps", "1", "--warmup", "0")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if "unavailable" in d:  # only when the engine could not be compiled here
        return
    assert d["metric"] == bench.METRIC and d["unit"] == "TOPS" and d["value"] > 0
    assert d["higher_is_better"] is True and d["steps"] == 1
    assert d["config"]["workload"] == bench.WORKLOAD
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "TOPS", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    p = run({"RANK": "1", "WORLD_SIZE": "2"}, "--impl", "reference", "--gpus", "2",
            "--steps", "1", "--warmup", "0")
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""
