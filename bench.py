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
decode kernels' achieved bandwidth to the measured HBM copy peak (a read+write copy;
a read-only kernel can exceed it, so `frac` may pass 1.0). `--impl reference`
times the reference algorithm's CPU path (the oracle's restatement of
decode_torch_optimized and the index-put append, float32) on the host cores.

Beside the headline (config 3) the same line carries, unless --headline-only:
  config4  the FP8 E4M3 per-tensor decode step (B=64 x 32768 tokens), measured the same
           way, with its own roofline and CPU baseline;
  config2  the KV append microbench (4096 new tokens) in each cache mode: device time
           per call from CUDA-graph replays over rotating input sets (12 x 16.8 MB of
           new K/V, more than L2, so every call reads its rows from HBM), roofline and
           the CPU baseline of the same append.
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
    ap.add_argument("--headline-only", action="store_true",
                    help="measure only --config (no config4 / config2 sub-records)")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch the step's decode after the append completes (no programmatic "
                         "dependent launch)")
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


def host_cpu():
    """CPU model, physical cores and logical CPUs of this host."""
    model = None
    phys = set()
    try:
        pid = core = None
        for line in open("/proc/cpuinfo"):
            k, _, v = line.partition(":")
            k, v = k.strip(), v.strip()
            if k == "model name" and model is None:
                model = v
            elif k == "physical id":
                pid = v
            elif k == "core id":
                core = v
            elif not k and pid is not None and core is not None:
                phys.add((pid, core))
                pid = core = None
        if pid is not None and core is not None:
            phys.add((pid, core))
    except OSError:
        pass
    logical = os.cpu_count() or 1
    try:
        affinity = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        affinity = logical
    physical = len(phys) if phys else logical
    return {"model": model, "physical_cores": physical, "logical_cpus": logical,
            "usable_cpus": affinity}


def cpu_threads() -> int:
    """Threads for the CPU baseline: the physical cores this process may run on."""
    h = host_cpu()
    return max(1, min(h["physical_cores"], h["usable_cpus"]))


def workload_config(args, world: int) -> dict:
    """The `config` object of the JSON line: the workload only (both arms print the same
    one), built from the BASELINE config's definition without touching a GPU."""
    if args.config == "config4":
        batch = args.batch or 64
        lens = [32768] * batch
        desc = "config4 (BASELINE config 4: FP8 decode, B=64, ctx 32768)"
    else:
        batch = args.batch or 256
        lens = torch.randint(1024, 8193, (batch,), generator=torch.Generator().manual_seed(0)).tolist()
        desc = "config3 (BASELINE config 3: bf16 decode, B=256, ctx U[1024,8192])"
    return {"workload": desc, "num_seqs": batch, "num_heads": 32, "num_kv_heads": 8,
            "head_dim": 128, "block_size": 256, "max_num_blocks": (max(lens) + 255) // 256,
            "parallelism": (f"kv-head tp{world}" if world > 1 else
                            f"rank 0 of a {args.emulate_shard}-way kv-head split, one GPU"
                            if args.emulate_shard > 1 else "single GPU"),
            "l2": "working set >> 126 MB L2 (no flush needed)",
            "step": "append 1 token/seq + paged decode"}


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


class Ranks:
    """Barrier, max/sum over ranks and CUDA-event timing on the launching stream."""

    def __init__(self, world: int, device):
        self.world, self.device = world, device
        self.stream = torch.cuda.current_stream(device)

    def barrier(self):
        if self.world > 1:
            dist.barrier()

    def _reduce(self, x: float, op) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], device=self.device, dtype=torch.float64)
        dist.all_reduce(t, op=op)
        return float(t)

    def max(self, x: float) -> float:
        return self._reduce(x, dist.ReduceOp.MAX if self.world > 1 else None)

    def sum(self, x: float) -> float:
        return self._reduce(x, dist.ReduceOp.SUM if self.world > 1 else None)

    def timed(self, fn, n: int) -> float:
        """ms per call of fn over n calls, events on the launching stream, synchronised
        and barriered on both sides."""
        self.barrier()
        torch.cuda.synchronize(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(n):
            fn()
        e1.record(self.stream)
        torch.cuda.synchronize(self.device)
        self.barrier()
        return e0.elapsed_time(e1) / n


class Replayer:
    """fn, or the replay of one CUDA graph of fn captured after a warm-up on a side
    stream (the reference's model runner replays its decode step from a captured graph,
    model_runner.py:690-704, 761-795). Graphs are kept until release()."""

    def __init__(self, device, eager: bool, warmup: int):
        self.device, self.eager, self.warmup = device, eager, max(3, warmup)
        self.graphs = []

    def __call__(self, fn):
        if self.eager:
            return fn
        dev = self.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        self.graphs.append(graph)
        for _ in range(self.warmup):
            graph.replay()
        torch.cuda.synchronize(dev)
        return graph.replay

    def release(self):
        torch.cuda.synchronize(self.device)
        self.graphs.clear()


def decode_step_fns(attn, w, ks, vs, overlap=True):
    fp8 = w.fp8

    def append(k=None, v=None, slots=None):
        k = w.new_k if k is None else k
        v = w.new_v if v is None else v
        slots = w.slot_mapping if slots is None else slots
        if fp8:
            attn.store_kvcache_fp8(k, v, w.k_cache, w.v_cache, ks, vs, slots, w.block_size,
                                   "fp8_per_tensor")
        else:
            attn.store_kvcache(k, v, w.k_cache, w.v_cache, slots, w.block_size)

    def decode(q=None, bt=None, cl=None, after_append=False):
        """after_append: the decode directly follows this step's append, so its prologue
        may overlap it (as Attention.forward runs them)."""
        q = w.query if q is None else q
        bt = w.block_tables if bt is None else bt
        cl = w.context_lens if cl is None else cl
        after_append = after_append and overlap
        if fp8:
            return attn.paged_attention_decode_quantized(
                q, w.k_cache, w.v_cache, ks, vs, bt, cl, w.scale, w.num_heads, w.num_kv_heads,
                w.head_dim, w.block_size, "fp8_per_tensor", overlap_previous=after_append)
        return attn.paged_attention_decode(q, w.k_cache, w.v_cache, bt, cl, w.scale, w.num_heads,
                                           w.num_kv_heads, w.head_dim, w.block_size,
                                           overlap_previous=after_append)

    return append, decode


def measure_e2e(args, w, append, decode, ranks, replay, total_step_bytes):
    """The step through the public API with host buffers: every step copies its inputs
    from pinned host memory and its output back, inside the timed region.

    The step's host inputs are packed into one pinned buffer (256-byte aligned parts), so
    that each step makes one host-to-device copy into a device buffer whose views are the
    step's input tensors. Two such buffers (each with its own captured step and output)
    let step i+1's input copy and step i-1's output copy run on copy streams while step i
    computes."""
    device, stream = ranks.device, ranks.stream
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
            append(dk, dv, ds)
            dout[:] = [decode(dq, dbt, dcl, after_append=True)]

        dbuf.copy_(hbuf)
        run = replay(device_part)
        hout = torch.empty(w.query.shape, dtype=w.query.dtype).pin_memory()
        return dbuf, run, dout, hout

    slots = [make_slot() for _ in range(2)]
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_steps(n_steps):
        ranks.barrier()
        torch.cuda.synchronize(device)
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
        torch.cuda.synchronize(device)
        ranks.barrier()
        return e0.elapsed_time(e1) / n_steps

    e2e_steps(4)
    e2e_ms = ranks.max(e2e_steps(args.steps))
    h2d = ranks.sum(hbuf.numel())
    d2h = ranks.sum(slots[0][3].numel() * slots[0][3].element_size())
    batch = w.query.shape[0]
    return {"value": round(total_step_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(e2e_ms, 4),
            "layer_decode_tokens_per_s": round(batch / (e2e_ms * 1e-3), 1),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)}


def measure_decode(args, cfg, rank, world, ranks, replay, attn, lib, headline: bool):
    """One decode config: the step (append + decode) replayed, then the decode and the
    append alone; e2e and clocks for the headline config."""
    device = ranks.device
    w = make_workload(cfg, rank, world, device, args.batch, args.emulate_shard)
    ks = w.k_scale.clone() if w.fp8 else None
    vs = w.v_scale.clone() if w.fp8 else None
    splits = lib.mkv_paged_decode_num_splits(w.query.shape[0], w.num_heads, w.num_kv_heads,
                                             w.head_dim, w.block_size, w.block_tables.shape[1])
    append, decode = decode_step_fns(attn, w, ks, vs, overlap=not args.no_overlap)

    def step():
        append()
        return decode(after_append=True)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)
    step_r, decode_r, append_r = replay(step), replay(decode), replay(append)

    clocks = None
    if headline:
        sampler = ClockSampler(ranks.device.index)
        with sampler:
            step_ms = ranks.timed(step_r, args.steps)
        clocks = sampler.summary() if rank == 0 else None
    else:
        step_ms = ranks.timed(step_r, args.steps)
    step_ms_max = ranks.max(step_ms)
    decode_ms = ranks.max(ranks.timed(decode_r, args.steps))
    append_ms = ranks.max(ranks.timed(append_r, args.steps))

    total_step_bytes = ranks.sum(w.decode_bytes() + w.append_bytes())
    total_decode_bytes = ranks.sum(w.decode_bytes())
    batch = w.query.shape[0]
    e2e = None
    if headline and not args.no_e2e:
        e2e = measure_e2e(args, w, append, decode, ranks, replay, total_step_bytes)
    peak, peak_kind = hbm_peak()
    achieved = total_decode_bytes / world / (decode_ms * 1e-3) / 1e9  # per GPU
    traffic = ncu_traffic(w.name, world)
    res = {
        "workload": w.name, "fp8": w.fp8, "batch": batch, "splits": splits,
        "num_heads": w.meta["num_heads"], "num_kv_heads": w.meta["num_kv_heads"],
        "head_dim": w.head_dim, "block_size": w.block_size,
        "max_num_blocks": w.block_tables.shape[1],
        "value": round(total_step_bytes / (step_ms_max * 1e-3) / 1e9, 2),
        "ms_per_step": round(step_ms_max, 4), "decode_ms": round(decode_ms, 4),
        "append_ms": round(append_ms, 4),
        "layer_decode_tokens_per_s": round(batch / (step_ms_max * 1e-3), 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "peak_kind": "read+write copy (a read-only kernel can exceed it)",
                     "kernel": "paged_decode (main + split merge), per GPU",
                     "traffic": traffic,
                     "algorithmic_bytes_per_launch": int(total_decode_bytes / world)},
        "kernels_per_step": 2,  # the append and the decode (its split merge is in-kernel)
        "e2e": e2e, "clocks": clocks,
    }
    replay.release()
    del w, step_r, decode_r, append_r
    torch.cuda.empty_cache()
    return res


APPEND_MODES = ("bf16", "fp8_per_tensor", "fp8_per_token_head", "int8_per_token_head")
APPEND_SETS = 12  # rotating input sets of 16.8 MB each: 201 MB of new K/V > 126 MB L2


def append_call(attn, mode, a, kc, vc, ks, vs):
    if mode == "bf16":
        attn.store_kvcache(a.key, a.value, kc, vc, a.slot_mapping, a.block_size)
    elif mode == "int8_per_token_head":
        attn.store_kvcache_int8(a.key, a.value, kc, vc, ks, vs, a.slot_mapping, a.block_size)
    else:
        attn.store_kvcache_fp8(a.key, a.value, kc, vc, ks, vs, a.slot_mapping, a.block_size, mode)


def append_cache(mode, a, device):
    shape = (a.num_blocks, a.block_size) + tuple(a.key.shape[1:])
    dt = {"bf16": torch.bfloat16, "int8_per_token_head": torch.int8}.get(mode, torch.float8_e4m3fn)
    kc = torch.zeros(shape, dtype=dt, device=device)
    vc = torch.zeros_like(kc)
    if mode == "bf16":
        return kc, vc, None, None
    if mode == "fp8_per_tensor":  # the sentinel: the first (warm-up) call calibrates
        return kc, vc, torch.ones(1, device=device), torch.ones(1, device=device)
    return kc, vc, torch.ones(shape[:3], device=device), torch.ones(shape[:3], device=device)


def append_algo_bytes(mode, a) -> int:
    cache_elem = 2 if mode == "bf16" else 1
    scale_bytes = 2 * a.key.shape[0] * a.key.shape[1] * 4 if "per_token_head" in mode else 0
    return a.bytes(cache_elem) + scale_bytes


def measure_append(args, ranks, replay, attn):
    """Config 2 in each cache mode: device ms per append call, from replays of one CUDA
    graph of APPEND_SETS calls over distinct input sets (each read from HBM)."""
    wlm = importlib.import_module(PKG + ".workloads")
    device = ranks.device
    sets = [wlm.config2(device=device, seed=i) for i in range(APPEND_SETS)]
    peak, peak_kind = hbm_peak()
    out = {}
    for mode in APPEND_MODES:
        kc, vc, ks, vs = append_cache(mode, sets[0], device)

        def calls():
            for a in sets:
                append_call(attn, mode, a, kc, vc, ks, vs)

        calls()  # eager warm-up (the FP8 per-tensor scale is calibrated here)
        torch.cuda.synchronize(device)
        run = replay(calls)
        ms = ranks.max(ranks.timed(run, max(5, args.steps)) / APPEND_SETS)
        algo = append_algo_bytes(mode, sets[0])
        gbs = algo / (ms * 1e-3) / 1e9
        out[mode] = {"us_per_call": round(ms * 1e3, 3), "value": round(gbs, 1), "unit": "GB/s",
                     "algorithmic_bytes": algo,
                     "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak,
                                  "unit": "GB/s", "frac": round(gbs / peak, 4),
                                  "peak_source": peak_kind,
                                  "traffic": ncu_traffic("config2-" + mode, 1)}}
        replay.release()
        del kc, vc, ks, vs, run
    del sets
    torch.cuda.empty_cache()
    return out


def cpu_append_baseline(reps: int = 20):
    """The reference's append on the host cores (oracle restatements of attention.py:7-64,
    the FP8 per-tensor quantiser 118-191 with the frozen scale, and the per-(token, head)
    quantisers), config 2, median of `reps` calls, in the same algorithmic GB/s."""
    from oracle import (store_kvcache_fp8_ref, store_kvcache_quant_per_token_head_ref,
                        store_kvcache_ref)
    wlm = importlib.import_module(PKG + ".workloads")
    threads = cpu_threads()
    torch.set_num_threads(threads)
    a = wlm.config2(device="cpu", seed=0)
    out = {}
    for mode in APPEND_MODES:
        kc, vc, ks, vs = append_cache(mode, a, "cpu")
        if mode == "bf16":
            fn = lambda: store_kvcache_ref(a.key, a.value, kc, vc, a.slot_mapping, a.block_size)
        elif mode == "fp8_per_tensor":
            fn = lambda: store_kvcache_fp8_ref(a.key, a.value, kc, vc, ks, vs, a.slot_mapping, a.block_size)
        else:
            m = mode.split("_")[0]
            fn = lambda: store_kvcache_quant_per_token_head_ref(a.key, a.value, kc, vc, ks, vs,
                                                                a.slot_mapping, a.block_size, m)
        fn()  # FP8 per tensor: calibrates here; the timed calls run with the frozen scale
        times = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        t = statistics.median(times)
        out[mode] = {"value": round(append_algo_bytes(mode, a) / t / 1e9, 3), "unit": "GB/s",
                     "us_per_call": round(t * 1e6, 1)}
    return {"kind": "port", "cores": threads, "host": host_cpu(),
            "sample": f"config 2 in full (4096 tokens), oracle restatement on {threads} threads, "
                      f"median of {reps} calls", "modes": out}


def run_ours(args, rank, world, local):
    mkv = importlib.import_module(PKG)
    attn = importlib.import_module(PKG + ".layers.attention")
    build = importlib.import_module(PKG + ".build")
    if rank == 0 and not build.up_to_date():
        build.build()  # never time a library compiled before the last source edit
    if world > 1:
        deadline = time.time() + 600
        while not build.up_to_date() and time.time() < deadline:
            time.sleep(1)
    lib = mkv.load()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    ranks = Ranks(world, device)
    replay = Replayer(device, args.eager, args.warmup)

    head = measure_decode(args, args.config, rank, world, ranks, replay, attn, lib, headline=True)
    subs = {}
    if not args.headline_only and args.batch == 0 and args.emulate_shard == 1:
        if args.config != "config4":
            subs["config4"] = measure_decode(args, "config4", rank, world, ranks, replay, attn, lib,
                                             headline=False)
        subs["config2"] = measure_append(args, ranks, replay, attn)

    # ---- CPU baselines (rank 0, N=1 only): the reference algorithm on the host cores
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(args.config, reps=5)
        if "config4" in subs:
            subs["config4"]["cpu_baseline"] = cpu_baseline_sample("config4", reps=3)
        if "config2" in subs:
            subs["config2"]["cpu_baseline"] = cpu_append_baseline()

    replay.release()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    fp8 = head["fp8"]
    line = {
        "metric": METRIC, "value": head["value"], "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp8_e4m3 cache, bf16 q/out, fp32 accumulate" if fp8 else "bf16 (fp32 accumulate)",
        "data": "synthetic (seeded N(0,1), random page permutation)",
        "config": workload_config(args, world),
        "method": {"num_splits": head["splits"],
                   "overlap": not args.no_overlap,
                   "launch": "eager" if args.eager else
                             "CUDA-graph replay of the step (e2e: one pinned H2D copy, replay, D2H copy per step, "
                             "copies of neighbouring steps overlapped on two copy streams)"},
        "layer_decode_tokens_per_s": head["layer_decode_tokens_per_s"],
        "layer_decode_tokens_per_s_note": "sequences per second through ONE attention layer's append + "
                                          "decode step; not model decode throughput",
        "append_ms": head["append_ms"], "decode_ms": head["decode_ms"],
        "e2e": head["e2e"],
        "roofline": head["roofline"],
        "gpu_launches": head["kernels_per_step"] * args.steps,
        "clocks": head["clocks"],
        "cpu_baseline": cpu,
        "build": {"library": "libmkv.so", "source_hash": lib.mkv_source_hash().decode(),
                  "version": lib.mkv_version().decode()},
    }
    for k, v in subs.items():
        if k == "config4":
            v = {kk: vv for kk, vv in v.items() if kk not in ("e2e", "clocks")}
        line[k] = v
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
    threads = cpu_threads()
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
            "cores": threads, "kind": "port", "host": host_cpu(),
            "sample": f"{nseq} sequences of {cfg} (all 32 heads), append + decode_torch_optimized "
                      f"restated in float32 on CPU, {threads} threads (one per physical core), "
                      f"median of {reps} ({t * 1e3:.1f} ms/sample)",
            "layer_decode_tokens_per_s": round(nseq / t, 2)}


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = cpu_threads()
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
              f"append + decode_torch_optimized restated in float32 on {threads} host threads "
              f"(one per physical core)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(total_t / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (reference CPU path)",
        "data": "synthetic (seeded N(0,1), random page permutation)",
        "config": workload_config(args, world),
        "layer_decode_tokens_per_s": round(total_seq / total_t, 2),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "host": host_cpu(), "sample": sample},
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
