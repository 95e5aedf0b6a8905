"""Paged decode over 8-bit caches with per-(token, head) scales ('fp8_per_token_head',
'int8_per_token_head'), at BASELINE config 3 and config 4 shapes, on one GPU.

    python mini-kvllm_b200/bench_decode_quant.py                        # the four cases
    python mini-kvllm_b200/bench_decode_quant.py --case config4,fp8_per_token_head --batch 8 \\
        --no-graph --launches 3                                         # a short run for profilers

Shapes:
- config 3: 256 sequences, H=32, KVH=8, D=128, 256-token pages, contexts U[1024, 8192];
- config 4: 64 sequences of 32768 tokens.

Pages hold seeded random bytes, finite for e4m3. Scales are seeded uniform in
[0.001, 0.021), and queries are bf16 N(0, 1). The algorithmic bytes per launch are:
- every visible token's K and V row (1 byte per element);
- its K and V scale (4 bytes each per kv head);
- the query read and the output write.
GB/s is that divided by the device time of one launch: CUDA-graph replays, CUDA events,
and the mean of `--iters`. The fraction is taken of the measured copy peak in
MEASURED_PEAKS.json when the file is present.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import sys

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(_HERE))
_PKG = os.path.basename(_HERE)
attn = importlib.import_module(_PKG + ".layers.attention")
wl = importlib.import_module(_PKG + ".workloads")
CASES = [(c, m) for c in ("config3", "config4") for m in ("fp8_per_token_head", "int8_per_token_head")]


def peak_gbs():
    path = os.path.join(os.path.dirname(_HERE), "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(path))["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="CONFIG,MODE")
    ap.add_argument("--batch", type=int, default=0, help="sequences (0: the config's)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--launches", type=int, default=3)
    args = ap.parse_args()
    cases = [tuple(args.case.split(","))] if args.case else CASES
    peak = peak_gbs()
    for cfg, mode in cases:
        kw = {"batch": args.batch} if args.batch else {}
        w = getattr(wl, cfg)(device="cuda", seed=0, with_append=False, **kw)
        NB, BS, KVH, D = w.k_cache.shape
        g = torch.Generator(device="cuda").manual_seed(1)
        bytes_ = torch.randint(-100, 100, (2, NB, BS, KVH, D), dtype=torch.int8, device="cuda", generator=g)
        if mode.startswith("fp8"):
            bytes_.view(torch.uint8).bitwise_and_(0x77)  # finite e4m3 values
            kc, vc = bytes_[0].view(torch.float8_e4m3fn), bytes_[1].view(torch.float8_e4m3fn)
        else:
            kc, vc = bytes_[0], bytes_[1]
        ks = torch.rand(NB, BS, KVH, device="cuda", generator=g) * 0.02 + 0.001
        vs = torch.rand(NB, BS, KVH, device="cuda", generator=g) * 0.02 + 0.001
        tokens = int(w.context_lens.clamp(max=w.block_tables.shape[1] * BS).sum())
        algo = tokens * KVH * (D * 2 + 4 * 2) + 2 * w.query.numel() * w.query.element_size()
        fn = lambda: attn.paged_attention_decode_quantized(
            w.query, kc, vc, ks, vs, w.block_tables, w.context_lens, w.scale, w.num_heads,
            w.num_kv_heads, w.head_dim, w.block_size, mode)
        if args.no_graph:
            for _ in range(args.launches):
                fn()
            torch.cuda.synchronize()
            print(json.dumps({"case": [cfg, mode], "launches": args.launches}))
        else:
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
            for _ in range(args.iters):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1) / args.iters * 1e-3
            gbs = algo / t / 1e9
            print(json.dumps({"case": [cfg, mode], "sequences": int(w.query.shape[0]), "us": round(t * 1e6, 1),
                              "algorithmic_bytes": algo, "GB/s": round(gbs, 1),
                              "frac_of_measured_peak": round(gbs / peak, 3) if peak else None}))
            del graph
        del w, kc, vc, ks, vs, bytes_
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
