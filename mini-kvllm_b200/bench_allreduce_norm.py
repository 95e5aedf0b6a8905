"""Tensor-parallel all-reduce + residual add + RMSNorm: the fused one-shot NVLink kernel
against NCCL all_reduce followed by the same residual add + RMSNorm.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        mini-kvllm_b200/bench_allreduce_norm.py [--check [--dump DIR]] [--hidden 1024] [--tokens 1,16,64]

One process per GPU, NCCL for the baseline and for exchanging the IPC handles.
- The partials are seeded per rank; the residual and the weight are shared.
- `--check` runs one fused call per token count and requires all ranks' outputs and sums
  to be bit-identical; it prints "check ok" on rank 0. With `--dump DIR` every rank also
  writes its inputs and results to DIR/rank<r>_T<T>.pt, for the test suite to compare with
  its CPU oracle.
- Timing, two ways, each the slowest rank's (max over ranks):
  - `*_us`: the median over `--iters` eager calls of the device time between CUDA events
    around each call. Host launch time is included whenever the GPU waits for it.
  - `*_graph_us`: 20 calls captured in one CUDA graph, replayed `--iters` / 20 times.
    This is the device time per call, as a runner that captures its decode step sees it.
  One JSON line per token count on rank 0.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

_HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(_HERE))
arn = importlib.import_module(os.path.basename(_HERE) + ".layers.allreduce_norm")


def timed(fn, iters: int) -> float:
    """Median device milliseconds of fn() over iters calls (events around each)."""
    ts = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ts.sort()
    return ts[len(ts) // 2]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--check", action="store_true")
    ap.add_argument("--dump", default="")
    ap.add_argument("--hidden", type=int, default=1024)
    ap.add_argument("--tokens", default="1,16,64,256,1024")
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--eps", type=float, default=1e-6)
    args = ap.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    H = args.hidden
    tokens = [int(t) for t in args.tokens.split(",")]
    ar = arn.AllReduceResidualRMSNorm(max(tokens), H, dtype=torch.bfloat16, timeout_ms=2000.0)
    g = torch.Generator(device=dev).manual_seed(1234)
    weight = (torch.rand(H, generator=g, device=dev) + 0.5).bfloat16()
    ok = True
    for T in tokens:
        gr = torch.Generator(device=dev).manual_seed(100 + rank * 7919 + T)
        partial = torch.randn(T, H, generator=gr, device=dev).bfloat16()
        gs = torch.Generator(device=dev).manual_seed(5 + T)
        residual0 = (torch.randn(T, H, generator=gs, device=dev) * 2).bfloat16()
        if args.check:
            buf = ar.next_partial(T)
            buf.copy_(partial)
            residual = residual0.clone()
            out, s = ar(buf, residual, weight, args.eps)
            ar.check()
            outs = [torch.empty_like(out) for _ in range(world)]
            sums = [torch.empty_like(s) for _ in range(world)]
            dist.all_gather(outs, out)
            dist.all_gather(sums, s)
            same = all(torch.equal(o, outs[0]) for o in outs) and all(torch.equal(x, sums[0]) for x in sums)
            if not same:
                print(f"rank {rank} T {T}: results differ across ranks", flush=True)
                ok = False
            if args.dump:
                torch.save({"partial": partial.cpu(), "residual": residual0.cpu(), "weight": weight.cpu(),
                            "eps": args.eps, "out": out.cpu(), "sum": s.cpu(), "world": world},
                           os.path.join(args.dump, f"rank{rank}_T{T}.pt"))
        # timing (every rank runs the same calls)
        residual = residual0.clone()
        buf = None

        def fused():
            nonlocal buf
            buf = ar.next_partial(T)  # the projection would write here; contents as left
            ar(buf, residual, weight, args.eps)

        nccl_buf = partial.clone()
        solo = arn.AllReduceResidualRMSNorm(T, H, dtype=torch.bfloat16)  # world-1 epilogue

        def baseline():
            dist.all_reduce(nccl_buf)
            solo(nccl_buf, residual, weight, args.eps)

        def baseline_torch():  # the reference's ops: NCCL, then torch add and RMSNorm
            dist.all_reduce(nccl_buf)
            x = nccl_buf + residual
            v = x.float().pow(2).mean(-1, keepdim=True) + args.eps
            (x.float() / v.sqrt() * weight.float()).bfloat16()

        for f in (fused, baseline, baseline_torch):
            for _ in range(10):
                f()
        torch.cuda.synchronize()
        dist.barrier()
        res = {}
        for name, f in (("fused_us", fused), ("nccl_plus_norm_us", baseline), ("nccl_plus_torch_us", baseline_torch)):
            dist.barrier()
            t = torch.tensor([timed(f, args.iters)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[name] = round(float(t.item()) * 1e3, 2)
        # CUDA graphs of 20 calls each (the NCCL one holds NCCL calls: released below,
        # before the process group is destroyed)
        for name, f in (("fused_graph_us", fused), ("nccl_plus_norm_graph_us", baseline)):
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                f()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(20):
                    f()
            graph.replay()
            torch.cuda.synchronize(dev)
            dist.barrier()
            reps = max(1, args.iters // 20)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            e1.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / (reps * 20)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[name] = round(float(t.item()) * 1e3, 2)
            del graph
            torch.cuda.synchronize(dev)
        ar.check()
        if rank == 0:
            print(json.dumps({"world": world, "tokens": T, "hidden": H, "dtype": "bf16", **res}), flush=True)
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    if args.check and rank == 0 and int(flag.item()) == 0:
        print("check ok", flush=True)
    ar.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(int(flag.item()))



if __name__ == "__main__":
    main()
