"""bench.py's reference arm on the CPU: one JSON line with the keys the measurement
contract names, and no output from ranks other than 0 (no GPU involved)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--steps", "3", "--warmup", "3"], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=600)


def test_reference_arm_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["steps"] == 3 and d["warmup"] == 3 and d["value"] > 0
    assert d["higher_is_better"] is True
    assert d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["cores"] >= 1
    assert cb["kind"] in ("reference", "port") and cb["sample"]
    e = d["e2e"]
    assert e == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_are_silent():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
