"""The benchmark's reference arm, `bench.py --impl reference`, on the CPU.

That arm times the reference algorithm's CPU path (the oracle restatement of the
index-put append and decode_torch_optimized, fp32) on a bounded sample of the config 3
workload. This test runs it as a user would: a subprocess with a short step count.
It checks the one JSON line against the output contract: metric, unit, the reference
marker, the CPU baseline block, the e2e block with zero copy bytes. It also checks that
ranks other than 0 exit without output."""
import json
import os
import subprocess
import sys

from conftest import REPO


def _run(env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
           "--warmup", "3"]
    return subprocess.run(["timeout", "-k", "10", "300"] + cmd, env=env, capture_output=True,
                          text=True, cwd=REPO)


def test_reference_arm_json_line():
    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["metric"].startswith("paged decode KV-cache HBM GB/s")
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] >= 3
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_nonzero_rank_is_silent():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
