"""Benchmark of the paged KV-cache decode step (append + paged-attention decode).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config config3|config4]
                    [--impl ours|reference]
    torchrun --nproc-per-node N ... bench.py --gpus N ...      (one rank per GPU)

Workload (default BASELINE config 3): Qwen3-8B attention shape, H=32 query heads,
KVH=8 KV heads, head_dim 128, block_size 256, batch 256, context lengths ~ U[1024, 8192],
random page permutation, bf16 q/K/V ~ N(0,1), synthetic and seeded. config4 is the FP8
E4M3 per-tensor cache at batch 64 x 32768 tokens. Under N ranks the KV heads are
sharded (rank r owns KV heads [r*8/N, (r+1)*8/N) and their query heads) with the full
batch on every rank: total work is fixed, so scaling is strong; the decode needs no
collective.

One step = what an attention layer does per decode step: append each sequence's new
K/V token into its page (store_kvcache / store_kvcache_fp8), then decode every
sequence over its whole context (paged_attention_decode[_quantized]). The step is
captured once in a CUDA graph and replayed, as the reference's model runner replays its
decode step; `--eager` times the Python calls instead.

Output: one JSON line from rank 0. `value` = algorithmic bytes of all ranks per step /
max-over-ranks step time, in GB/s (K/V cache reads dominate; the working set of
config 3 is ~5 GB, far larger than the 126 MB L2, so no flush is needed). `e2e` is the
same metric through the public API with the step's inputs copied from pinned host
memory and the output copied back inside the timed region. `roofline` relates the
decode kernels' achieved bandwidth to the measured HBM copy peak. `--impl reference`
times the reference algorithm's CPU path (the oracle's restatement of
decode_torch_optimized and the index-put append, float32) on the host cores.
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
PKG = "mini-kvllm_b200"

METRIC = "paged decode KV-cache HBM GB/s (% of roofline) and decode tokens/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="config3", choices=["config3", "config4"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the number of sequences (smaller cases for ncu captures)")
    ap.add_argument("--emulate-shard", type=int, default=1,
                    help="run rank 0's KV-head shard of an N-way split on this one GPU")
    ap.add_argument("--eager", action="store_true",
                    help="time eager launches instead of CUDA-graph replays of the step")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def hbm_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(workload: str, world: int):
    """DRAM bytes per decode launch from the committed ncu summary, when one exists for
    this workload and shard count (a line `ncu-traffic <workload> <world> <bytes>`)."""
    pdir = os.path.join(REPO, "profiles")
    if not os.path.isdir(pdir):
        return None
    pat = re.compile(r"^ncu-traffic\s+(\S+)\s+(\d+)\s+([0-9.eE+]+)\s*$")
    for name in sorted(os.listdir(pdir)):
        if not name.endswith((".md", ".txt")):
            continue
        with open(os.path.join(pdir, name)) as f:
            for line in f:
                m = pat.match(line.strip().strip("`"))
                if m and m.group(1) == workload and int(m.group(2)) == world:
                    return float(m.group(3))
    return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"mkv_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()
        return False

    def summary(self):
        if self.proc is None:
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
            os.unlink(self.path)
        except Exception:
            return None
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_workload(cfg: str, rank: int, world: int, device, batch: int = 0, shard: int = 1):
    wl = importlib.import_module(PKG + ".workloads")
    kw = {"batch": batch} if batch > 0 else {}
    if world == 1 and shard > 1:  # one rank's shard of an N-way split, on one GPU
        rank, world = 0, shard
    return getattr(wl, cfg)(device=device, seed=0, rank=rank, world_size=world, **kw)


def run_ours(args, rank, world, local):
    mkv = importlib.import_module(PKG)
    attn = importlib.import_module(PKG + ".layers.attention")
    lib = mkv.load()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))

    w = make_workload(args.config, rank, world, device, args.batch, args.emulate_shard)
    fp8 = w.fp8
    ks = w.k_scale.clone() if fp8 else None
    vs = w.v_scale.clone() if fp8 else None
    splits = lib.mkv_paged_decode_num_splits(w.query.shape[0], w.num_heads, w.num_kv_heads,
                                             w.head_dim, w.block_size, w.block_tables.shape[1])

    def append():
        if fp8:
            attn.store_kvcache_fp8(w.new_k, w.new_v, w.k_cache, w.v_cache, ks, vs, w.slot_mapping,
                                   w.block_size, "fp8_per_tensor")
        else:
            attn.store_kvcache(w.new_k, w.new_v, w.k_cache, w.v_cache, w.slot_mapping, w.block_size)

    def decode(q=None, bt=None, cl=None):
        q = w.query if q is None else q
        bt = w.block_tables if bt is None else bt
        cl = w.context_lens if cl is None else cl
        if fp8:
            return attn.paged_attention_decode_quantized(
                q, w.k_cache, w.v_cache, ks, vs, bt, cl, w.scale, w.num_heads, w.num_kv_heads,
                w.head_dim, w.block_size, "fp8_per_tensor")
        return attn.paged_attention_decode(q, w.k_cache, w.v_cache, bt, cl, w.scale, w.num_heads,
                                           w.num_kv_heads, w.head_dim, w.block_size)

    def step():
        append()
        return decode()

    stream = torch.cuda.current_stream()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    def replayed(fn):
        """fn, or a replay of one CUDA graph of fn (the reference's model runner replays
        its decode step from a captured graph, model_runner.py:690-704, 761-795)."""
        if args.eager:
            return fn
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        graphs.append(graph)
        for _ in range(max(3, args.warmup)):
            graph.replay()
        torch.cuda.synchronize(device)
        return graph.replay

    graphs = []
    step_r, decode_r, append_r = replayed(step), replayed(decode), replayed(append)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t)
        return float(t)

    def timed(fn, n):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1) / n  # ms

    # ---- device-resident step (the headline `value`), clocks sampled meanwhile
    sampler = ClockSampler(local)
    with sampler:
        step_ms = timed(step_r, args.steps)
    clocks = sampler.summary() if rank == 0 else None
    step_ms_max = max_over_ranks(step_ms)

    # ---- the dominant kernel(s) alone: decode (main kernel + split merge)
    decode_ms = max_over_ranks(timed(decode_r, args.steps))
    append_ms = max_over_ranks(timed(append_r, args.steps))

    step_bytes = w.decode_bytes() + w.append_bytes()
    total_step_bytes = sum_over_ranks(step_bytes)
    total_decode_bytes = sum_over_ranks(w.decode_bytes())
    batch = w.query.shape[0]
    value = total_step_bytes / (step_ms_max * 1e-3) / 1e9
    tokens_per_s = batch / (step_ms_max * 1e-3)

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        # The step's host inputs packed into one pinned buffer (256-byte aligned parts),
        # so that each step makes one host-to-device copy into a device buffer whose
        # views are the step's input tensors. Two such buffers (each with its own
        # captured step and output) let step i+1's input copy and step i-1's output copy
        # run on copy streams while step i computes; every step still copies its inputs
        # in and its output out inside the timed region.
        srcs = (w.query, w.new_k, w.new_v, w.slot_mapping, w.block_tables, w.context_lens)
        offs, n = [], 0
        for t in srcs:
            offs.append(n)
            n += (t.numel() * t.element_size() + 255) // 256 * 256
        hbuf = torch.empty(n, dtype=torch.uint8).pin_memory()

        def part(buf, t, off):
            nb = t.numel() * t.element_size()
            return buf[off:off + nb].view(t.dtype).view(t.shape)

        for t, off in zip(srcs, offs):
            part(hbuf, t, off).copy_(t.cpu())

        def make_slot():
            dbuf = torch.empty(n, dtype=torch.uint8, device=device)
            dq, dk, dv, ds, dbt, dcl = (part(dbuf, t, off) for t, off in zip(srcs, offs))
            dout = []

            def device_part():  # append + decode on this slot's device input views
                if fp8:
                    attn.store_kvcache_fp8(dk, dv, w.k_cache, w.v_cache, ks, vs, ds, w.block_size,
                                           "fp8_per_tensor")
                else:
                    attn.store_kvcache(dk, dv, w.k_cache, w.v_cache, ds, w.block_size)
                dout[:] = [decode(dq, dbt, dcl)]

            dbuf.copy_(hbuf)
            run = replayed(device_part)
            hout = torch.empty(w.query.shape, dtype=w.query.dtype).pin_memory()
            return dbuf, run, dout, hout

        slots = [make_slot() for _ in range(2)]
        copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_used = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]

        def e2e_steps(n_steps):
            """n_steps end-to-end steps; returns the device ms per step (events on the
            launching stream around all of them, copy streams joined before the end)."""
            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            copy_in.wait_stream(stream)
            copy_out.wait_stream(stream)
            for i in range(n_steps):
                k = i % 2
                dbuf, run, dout, hout = slots[k]
                if i >= 2:
                    copy_in.wait_event(ev_used[k])  # step i-2 no longer reads this buffer
                with torch.cuda.stream(copy_in):
                    dbuf.copy_(hbuf, non_blocking=True)
                ev_in[k].record(copy_in)
                stream.wait_event(ev_in[k])
                if i >= 2:
                    stream.wait_event(ev_out[k])  # step i-2's output has been copied out
                run()
                ev_used[k].record(stream)
                copy_out.wait_event(ev_used[k])
                with torch.cuda.stream(copy_out):
                    hout.copy_(dout[0], non_blocking=True)
                if args.eager:  # a fresh output each call: keep it alive for the copy stream
                    dout[0].record_stream(copy_out)
                ev_out[k].record(copy_out)
            stream.wait_stream(copy_out)
            e1.record(stream)
            torch.cuda.synchronize()
            barrier()
            return e0.elapsed_time(e1) / n_steps

        e2e_steps(4)
        e2e_ms = max_over_ranks(e2e_steps(args.steps))
        h2d = sum_over_ranks(hbuf.numel())
        d2h = sum_over_ranks(slots[0][3].numel() * slots[0][3].element_size())
        e2e = {"value": round(total_step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(e2e_ms, 4), "decode_tokens_per_s": round(batch / (e2e_ms * 1e-3), 1),
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)}

    peak, peak_kind = hbm_peak()
    achieved = total_decode_bytes / world / (decode_ms * 1e-3) / 1e9  # per GPU
    traffic = ncu_traffic(w.name, world)
    kernels_per_step = (2 if fp8 else 1) + 1 + (1 if splits > 1 else 0)

    # ---- CPU baseline (rank 0, N=1 only): the reference algorithm on the host cores
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(args.config, reps=5)

    graphs.clear()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(step_ms_max, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp8_e4m3 cache, bf16 q/out, fp32 accumulate" if fp8 else "bf16 (fp32 accumulate)",
        "data": "synthetic (seeded N(0,1), random page permutation)",
        "config": {"workload": w.name + (" (BASELINE config 4: FP8 decode, B=64, ctx 32768)" if fp8 else
                                         " (BASELINE config 3: bf16 decode, B=256, ctx U[1024,8192])"),
                   "num_seqs": batch, "num_heads": w.meta["num_heads"], "num_kv_heads": w.meta["num_kv_heads"],
                   "head_dim": w.head_dim, "block_size": w.block_size,
                   "max_num_blocks": w.block_tables.shape[1], "num_splits": splits,
                   "parallelism": (f"kv-head tp{world}" if world > 1 else
                                   f"rank 0 of a {args.emulate_shard}-way kv-head split, one GPU"
                                   if args.emulate_shard > 1 else "single GPU"),
                   "l2": "working set >> 126 MB L2 (no flush needed)",
                   "step": "append 1 token/seq + paged decode",
                   "launch": "eager" if args.eager else
                             "CUDA-graph replay of the step (e2e: one pinned H2D copy, replay, D2H copy per step, "
                             "copies of neighbouring steps overlapped on two copy streams)"},
        "decode_tokens_per_s": round(tokens_per_s, 1),
        "append_ms": round(append_ms, 4), "decode_ms": round(decode_ms, 4),
        "e2e": e2e,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "kernel": "paged_decode (main + split merge), per GPU",
                     "traffic": traffic,
                     "algorithmic_bytes_per_launch": int(total_decode_bytes / world)},
        "gpu_launches": kernels_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


def _cpu_sample_workload(cfg: str, nseq: int, offset: int):
    """The first `offset + nseq` sequences of the workload, built on the CPU in float32
    (the reference's CPU path runs in fp32)."""
    wl = importlib.import_module(PKG + ".workloads")
    g = torch.Generator().manual_seed(0)
    if cfg == "config3":
        lens = torch.randint(1024, 8193, (256,), generator=g).tolist()
        fp8 = False
    else:
        lens = [32768] * 64
        fp8 = True
    lens = [lens[(offset + i) % len(lens)] for i in range(nseq)]
    w = wl.decode_workload(cfg + "-cpu-sample", nseq, 32, 8, 128, 256, lens, dtype=torch.float32,
                           fp8=fp8, device="cpu", seed=offset + 1)
    return w


def _cpu_step(w):
    from oracle import decode_torch_optimized, store_kvcache_ref
    kc, vc = w.k_cache, w.v_cache
    if w.fp8:  # dequantise-then-attend, as the reference's FP8 comparison does
        kc = kc.float() * float(w.k_scale)
        vc = vc.float() * float(w.v_scale)
    store_kvcache_ref(w.new_k, w.new_v, kc, vc, w.slot_mapping, w.block_size)
    return decode_torch_optimized(w.query, kc, vc, w.block_tables, w.context_lens, w.scale,
                                  w.num_heads, w.num_kv_heads, w.head_dim, w.block_size)


def _sample_bytes(w, cache_elem: int):
    """Algorithmic bytes of the sample counted at the GPU workload's element sizes."""
    tokens = int(w.context_lens.sum())
    kvh, d = w.num_kv_heads, w.head_dim
    q = w.query.numel() * 2
    return tokens * kvh * d * cache_elem * 2 + 2 * q + 2 * w.new_k.numel() * (2 + cache_elem)


def cpu_baseline_sample(cfg: str, reps: int = 5):
    nseq = 4 if cfg == "config3" else 1  # one 32k-token FP8 sequence pads to ~2 GB on the CPU
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = _cpu_sample_workload(cfg, nseq, 0)
    cache_elem = 1 if w.fp8 else 2
    _cpu_step(w)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        _cpu_step(w)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(_sample_bytes(w, cache_elem) / t / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "sample": f"{nseq} sequences of {cfg} (all 32 heads), append + decode_torch_optimized "
                      f"restated in float32 on CPU, median of {reps} ({t * 1e3:.1f} ms/sample)",
            "decode_tokens_per_s": round(nseq / t, 2)}


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    nseq = 4 if args.config == "config3" else 1
    samples = [_cpu_sample_workload(args.config, nseq, 4 * i) for i in range(2)]
    cache_elem = 1 if samples[0].fp8 else 2
    for i in range(max(3, args.warmup)):
        _cpu_step(samples[i % 2])
    total_t, total_b, total_seq = 0.0, 0, 0
    for i in range(args.steps):
        w = samples[i % 2]
        t0 = time.perf_counter()
        _cpu_step(w)
        total_t += time.perf_counter() - t0
        total_b += _sample_bytes(w, cache_elem)
        total_seq += nseq
    value = total_b / total_t / 1e9
    sample = (f"each step: {nseq} sequences of {args.config} (all 32 heads, full contexts), "
              f"append + decode_torch_optimized restated in float32 on {threads} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(total_t / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (reference CPU path)",
        "data": "synthetic (seeded N(0,1), random page permutation)",
        "config": {"workload": args.config, "cpu_sample_sequences_per_step": nseq},
        "decode_tokens_per_s": round(total_seq / total_t, 2),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit(f"--gpus {args.gpus} needs torchrun with {args.gpus} processes")
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
