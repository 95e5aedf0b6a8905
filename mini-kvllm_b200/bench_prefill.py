"""Chunked-prefill / extend throughput of `paged_attention_prefill` on one GPU.

    python mini-kvllm_b200/bench_prefill.py                  # the standard cases
    python mini-kvllm_b200/bench_prefill.py --case 2,2048,2048 --launches 3 --no-graph

Each case is (sequences, cached prefix tokens, chunk tokens): every sequence appends a
chunk of query tokens after its prefix, so query position p sees min(p + 1, context)
cached tokens. H=32 query heads, 8 KV heads, head_dim 128, 256-token pages in a random
order per sequence, bf16 queries; the cache is bf16, e4m3 with a per-tensor scale or
per-(token, head) scales, or int8 with per-(token, head) scales. Inputs are synthetic
(seeded normal values).

Throughput counts 4 · Σ visible tokens · H · D FLOPs per call, the work of QKᵀ and PV
over the visible tokens only, and times CUDA-graph replays with CUDA events. One JSON
line per case. `--no-graph --launches N` runs N plain calls instead (a short command for
profilers).
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import sys

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(_HERE))
attn = importlib.import_module(os.path.basename(_HERE) + ".layers.attention")

H, KVH, D, BS = 32, 8, 128, 256
CASES = [(8, 0, 2048, "auto"), (8, 4096, 2048, "auto"), (4, 16384, 4096, "auto"),
         (8, 4096, 2048, "fp8_per_tensor"), (8, 4096, 2048, "fp8_per_token_head"),
         (8, 4096, 2048, "int8_per_token_head")]


def make(nseq: int, prefix: int, chunk: int, mode: str, seed: int = 0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ctx = prefix + chunk
    nbs = (ctx + BS - 1) // BS
    nb = nseq * nbs
    bt = torch.stack([torch.randperm(nbs, device="cuda", generator=g) for _ in range(nseq)])
    bt = (bt + torch.arange(nseq, device="cuda").view(-1, 1) * nbs).to(torch.int32)
    cl = torch.full((nseq,), ctx, dtype=torch.int64, device="cuda")
    cu = torch.arange(0, (nseq + 1) * chunk, chunk, dtype=torch.int32, device="cuda")
    pos = torch.arange(prefix, ctx, device="cuda").repeat(nseq)
    q = torch.randn(nseq * chunk, H, D, device="cuda", generator=g).to(torch.bfloat16)
    kw = {}
    shape = (nb, BS, KVH, D)
    if mode == "auto":
        kc = torch.randn(shape, device="cuda", generator=g).to(torch.bfloat16)
        vc = torch.randn(shape, device="cuda", generator=g).to(torch.bfloat16)
    elif mode == "fp8_per_tensor":
        kc = (torch.randn(shape, device="cuda", generator=g) * 40).to(torch.float8_e4m3fn)
        vc = (torch.randn(shape, device="cuda", generator=g) * 40).to(torch.float8_e4m3fn)
        kw = dict(k_scale=torch.full((1,), 0.025, device="cuda"), v_scale=torch.full((1,), 0.025, device="cuda"),
                  kv_cache_dtype=mode)
    else:
        if mode == "fp8_per_token_head":
            kc = (torch.randn(shape, device="cuda", generator=g) * 40).to(torch.float8_e4m3fn)
            vc = (torch.randn(shape, device="cuda", generator=g) * 40).to(torch.float8_e4m3fn)
        else:
            kc = torch.randint(-127, 128, shape, device="cuda", generator=g, dtype=torch.int8)
            vc = torch.randint(-127, 128, shape, device="cuda", generator=g, dtype=torch.int8)
        kw = dict(k_scale=torch.rand(nb, BS, KVH, device="cuda", generator=g) * 0.02,
                  v_scale=torch.rand(nb, BS, KVH, device="cuda", generator=g) * 0.02, kv_cache_dtype=mode)
    vis = nseq * sum(min(ctx, p + 1) for p in range(prefix, ctx))
    fn = lambda: attn.paged_attention_prefill(q, kc, vc, bt, cl, cu, pos, 1.0 / math.sqrt(D), H, KVH, D, BS, **kw)
    return fn, 4.0 * vis * H * D


def time_graph(fn, iters: int) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e-3


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="SEQS,PREFIX,CHUNK[,MODE] (default: the standard cases)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--launches", type=int, default=3)
    args = ap.parse_args()
    cases = CASES
    if args.case:
        f = args.case.split(",")
        cases = [(int(f[0]), int(f[1]), int(f[2]), f[3] if len(f) > 3 else "auto")]
    for nseq, prefix, chunk, mode in cases:
        fn, flops = make(nseq, prefix, chunk, mode)
        if args.no_graph:
            for _ in range(args.launches):
                fn()
            torch.cuda.synchronize()
            print(json.dumps({"case": [nseq, prefix, chunk, mode], "launches": args.launches}))
            continue
        t = time_graph(fn, args.iters)
        print(json.dumps({"case": [nseq, prefix, chunk, mode], "ms": round(t * 1e3, 4),
                          "tflops": round(flops / t / 1e12, 1),
                          "qtiles": os.environ.get("MKV_PREFILL_QTILES", "auto")}))
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
