"""KV append + quantise at BASELINE config 2, on one GPU.

    python mini-kvllm_b200/bench_append.py                  # the four cache modes
    python mini-kvllm_b200/bench_append.py --mode fp8_per_tensor --iters 3   # for profilers

The workload is config 2: 4096 new tokens, 8 KV heads x head_dim 128, bf16 K/V ~ N(0,1)
with 0.1 % outliers x20. The tokens are 16 prefill chunks of 128 consecutive slots plus
2048 single tokens on random slots, in a 65536-slot paged cache (256 pages of 256).
Each mode is one append call through the Python API:
- bf16: store_kvcache into bf16 pages;
- fp8_per_tensor: store_kvcache_fp8, with the scale calibrated by the first (untimed)
  call. A timed call is one launch that reads the (frozen) scale and quantises;
- fp8_per_token_head / int8_per_token_head: one scale per (token, head) row, written
  beside the pages.

The working set (~34 MB) fits in the 126 MB L2. So a 512 MB buffer is written before
every timed call, and only the call sits between its CUDA events (the Python launch
included; bench.py's config2 record times graph replays instead). The mean over
`--iters` calls is reported. Used for ncu captures of the append kernels.

Algorithmic bytes per call:
- read: K and V in bf16, plus the int64 slots;
- write: K and V at the cache's element size, plus the two fp32 scales per row in the
  per-(token, head) modes.
GB/s is those bytes over the device time, and the fraction is taken of the measured
copy peak in MEASURED_PEAKS.json.
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
MODES = ("bf16", "fp8_per_tensor", "fp8_per_token_head", "int8_per_token_head")


def peak_gbs():
    path = os.path.join(os.path.dirname(_HERE), "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(path))["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return None


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", default=None, choices=MODES)
    ap.add_argument("--iters", type=int, default=50)
    args = ap.parse_args()
    peak = peak_gbs()
    w = wl.config2(device="cuda", seed=0)
    T, KVH, D = w.key.shape
    shape = (w.num_blocks, w.block_size, KVH, D)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    for mode in ([args.mode] if args.mode else MODES):
        if mode == "bf16":
            kc, vc = torch.zeros(shape, dtype=torch.bfloat16, device="cuda"), torch.zeros(shape, dtype=torch.bfloat16, device="cuda")
            call = lambda: attn.store_kvcache(w.key, w.value, kc, vc, w.slot_mapping, w.block_size)
            cache_elem, scale_bytes = 2, 0
        elif mode == "fp8_per_tensor":
            kc = torch.zeros(shape, dtype=torch.float8_e4m3fn, device="cuda")
            vc = torch.zeros_like(kc)
            ks, vs = torch.ones(1, device="cuda"), torch.ones(1, device="cuda")  # 1.0: calibrate
            call = lambda: attn.store_kvcache_fp8(w.key, w.value, kc, vc, ks, vs, w.slot_mapping,
                                                  w.block_size, "fp8_per_tensor")
            cache_elem, scale_bytes = 1, 0
        else:
            dt = torch.float8_e4m3fn if mode.startswith("fp8") else torch.int8
            kc = torch.zeros(shape, dtype=dt, device="cuda")
            vc = torch.zeros_like(kc)
            ks = torch.zeros(shape[:3], device="cuda")
            vs = torch.zeros_like(ks)
            if mode.startswith("fp8"):
                call = lambda: attn.store_kvcache_fp8(w.key, w.value, kc, vc, ks, vs, w.slot_mapping,
                                                      w.block_size, "fp8_per_token_head")
            else:
                call = lambda: attn.store_kvcache_int8(w.key, w.value, kc, vc, ks, vs, w.slot_mapping,
                                                       w.block_size)
            cache_elem, scale_bytes = 1, 2 * T * KVH * 4
        algo = w.bytes(cache_elem) + scale_bytes
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(args.iters):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            call()
            e1.record()
            e1.synchronize()
            total += e0.elapsed_time(e1)
        t = total / args.iters * 1e-3
        gbs = algo / t / 1e9
        print(json.dumps({"mode": mode, "tokens": T, "us": round(t * 1e6, 2), "algorithmic_bytes": algo,
                          "GB/s": round(gbs, 1),
                          "frac_of_measured_peak": round(gbs / peak, 3) if peak else None,
                          "l2": "512 MB written before each call"}), flush=True)
        del kc, vc
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
