"""The reference's own serving engine with this library's Attention dropped in.

mini-kvllm_b200/bench_engine.py drives the reference's ModelRunner and Scheduler
(installed in baseline/_ref) on a random-init Qwen3-0.6B-shaped model; with --impl ours
the model's Attention layers are this library's. A short run with an FP8 per-tensor
cache goes through the runner's warm-up (whole-prompt prefill before a cache exists),
chunked prefill mixed with decode, and pure decode steps, and must generate every
requested token. Skipped when the reference is not installed.
"""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu
REF_DIR = os.path.join(REPO, "baseline", "_ref")


@pytest.mark.parametrize("kv", ["fp8_per_tensor", "int8_per_token_head"])
def test_reference_engine_runs_with_libmkv_attention(kv):
    if not os.path.isdir(os.path.join(REF_DIR, "myvllm")):
        pytest.skip("reference not installed in baseline/_ref")
    cmd = [sys.executable, os.path.join(REPO, "mini-kvllm_b200", "bench_engine.py"), "--tp", "1",
           "--impl", "ours", "--kv", kv, "--requests", "12", "--output", "6", "--prompt-min", "100",
           "--prompt-max", "700", "--batched-tokens", "2048", "--max-seqs", "16",
           "--port", "29611" if kv.startswith("fp8") else "29612"]
    r = subprocess.run(["timeout", "-k", "10", "900"] + cmd, capture_output=True, text=True, cwd=REPO)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert lines, r.stdout[-2000:]
    d = json.loads(lines[-1])
    assert d["impl"] == "ours" and d["kv_cache_dtype"] == kv
    assert d["generated_tokens"] == 12 * 6
    assert d["decode_steps"] > 0 and d["tokens_per_s"] > 0
