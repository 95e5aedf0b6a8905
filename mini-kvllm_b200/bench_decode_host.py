"""Host cost of building one decode step's metadata (ModelRunner.prepare_decode,
model_runner.py:631-671) for BASELINE config 3's batch: 256 sequences, 256-token pages,
contexts U[1024, 8192] (up to 32 pages).

    python mini-kvllm_b200/bench_decode_host.py [--steps 200]

Two ways:
- `prepare_decode_style`: `decode_metadata`, which does what the reference does. It loops
  over the sequences in Python and makes three tensors, copied from pinned memory.
- `builder`: DecodeMetadataBuilder. It keeps the tables, packs the lengths, makes one
  copy and launches one kernel.
Per way: `host_us`, the host time per step (perf_counter, no synchronisation inside the
loop), and `wall_us`, the time per step until the GPU work of all steps has finished.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import random
import sys
import time

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(_HERE))
kvc = importlib.import_module(os.path.basename(_HERE) + ".engine.kv_cache")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=200)
    args = ap.parse_args()
    rng = random.Random(0)
    B, BS, W = 256, 256, 32
    lens = [rng.randint(1024, 8192) for _ in range(B)]
    perm = list(range(B * W))
    rng.shuffle(perm)
    tables = [perm[b * W: b * W + (n + BS - 1) // BS] for b, n in enumerate(lens)]
    builder = kvc.DecodeMetadataBuilder(B, W, BS)
    for b in range(B):
        builder.set_table(b, tables[b])
    seqs = list(range(B))
    out = {}
    for name, fn in (("prepare_decode_style", lambda: kvc.decode_metadata(tables, lens, BS, pin_memory=True)),
                     ("builder", lambda: builder.step(seqs, lens))):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        t1 = time.perf_counter()
        torch.cuda.synchronize()
        t2 = time.perf_counter()
        out[name] = {"host_us": round((t1 - t0) / args.steps * 1e6, 1),
                     "wall_us": round((t2 - t0) / args.steps * 1e6, 1)}
    print(json.dumps({"batch": B, "block_size": BS, "max_blocks": W, **out}))


if __name__ == "__main__":
    main()
