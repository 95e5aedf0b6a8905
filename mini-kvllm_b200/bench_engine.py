"""model decode tokens/s through the reference's own serving engine.

    python mini-kvllm_b200/bench_engine.py --tp N [--impl ours|reference] [--kv fp8_per_tensor]
                                           [--requests 256] [--output 256]

The reference (heart1128/mini-kvllm) must be installed in baseline/_ref (pip install
--target); its engine runs unmodified: ModelRunner (model_runner.py) with its warm-up,
KV-cache allocation and shared-memory RPC to the tensor-parallel workers, Scheduler
(scheduler.py) with chunked prefill mixed into decode batches, its Qwen3 model, sampler
and NCCL all-reduces. What this script changes, and only at import time in every rank:
  * weights: no checkpoint or network here, so load_weights_from_checkpoint (utils/
    loader.py) is replaced by a seeded random initialisation of the same parameters
    (std 0.02, norms 1), and prompts are random token ids fed to the scheduler as
    Sequence objects (no tokenizer);
  * --impl ours: the model's Attention layer (attention.py:1617-1807) is this library's
    Attention, which reads the reference's context (utils/context.py), appends with
    libmkv's store kernels and runs libmkv's prefill and decode kernels;
    --impl reference keeps the reference's Triton attention. The reference raises
    NotImplementedError for chunked prefill over a quantised cache (attention.py:
    1702-1708), so its arm uses kv 'auto' unless told otherwise.
  * the model runs in bf16 (torch.set_default_dtype), as config 5 names; the reference
    would otherwise build fp32 parameters, and its RoPE returns float32 q/k for bf16
    inputs (a float32 cos/sin cache), so RoPE's outputs are cast back to bf16.
  * tensor parallelism (TP > 1): the reference's Sequence pickles a compact state for
    the workers (sequence.py:98-130) that leaves out block_size and, in decode, all but
    the last token id, so a worker's prepare_decode (model_runner.py:639) raises at
    sequence.py:81 whatever the attention. block_size is restored on unpickling and the
    last block's token count is taken from num_tokens, the value rank 0 computes from
    its full token list (both arms alike).
Workload (config 5, synthetic and seeded): Qwen3-0.6B shape (28 layers, hidden 1024,
16 Q / 8 KV heads, head_dim 128, MLP 3072, vocab 151936); --requests prompts of random
token ids with lengths ~ U[128, 1024]; --output tokens each (ignore_eos: random weights
would otherwise end sequences at random) at temperature 0.6; enforce_eager as in the
reference's own benchmarks (its graph capture reads a config key they never set).

Output: one JSON line from rank 0. tokens_per_s = generated tokens / wall time of the
whole run (prefill included); decode_tokens_per_s = tokens sampled in decode-only steps
/ the wall time of those steps.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import time

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(_HERE)
PKG = os.path.basename(_HERE)
REF_DIR = os.path.join(REPO, "baseline", "_ref")
for p in (REPO, REF_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def qwen3_0p6b_config(tp: int, kv: str, max_model_length: int, batched_tokens: int,
                      max_seqs: int, port: int) -> dict:
    return {
        "max_num_sequences": max_seqs, "max_num_batched_tokens": batched_tokens,
        "max_cached_blocks": 4096, "block_size": 256, "world_size": tp,
        "model_name_or_path": "Qwen3-0.6B", "enforce_eager": True,
        "vocab_size": 151936, "hidden_size": 1024, "num_heads": 16, "head_dim": 128,
        "num_kv_heads": 8, "intermediate_size": 3072, "num_layers": 28,
        "tie_word_embeddings": True, "base": 1000000, "rms_norm_epsilon": 1e-6,
        "qkv_bias": False, "scale": 1, "max_position": 32768, "ffn_bias": False,
        "max_num_batch_tokens": batched_tokens, "max_model_length": max_model_length,
        "gpu_memory_utilization": 0.85, "eos": 151645, "kv_cache_dtype": kv,
        "bench_port": port,
    }


def random_weights(model, path):  # replaces load_weights_from_checkpoint(model, path)
    """Seeded random parameters of the checkpoint's shapes: normal(0, 0.02) for matrices
    and embeddings, 1 for norm weights, 0 for biases (per rank: each holds its shard)."""
    rank = torch.distributed.get_rank() if torch.distributed.is_initialized() else 0
    g = torch.Generator(device="cpu").manual_seed(1234 + rank)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                cpu = torch.empty(p.shape, dtype=torch.float32, device="cpu").normal_(0.0, 0.02, generator=g)
                p.copy_(cpu)


def sequence_state_for_workers(block_size: int) -> None:
    """Make the reference's Sequence usable on tensor-parallel workers: restore
    block_size when a Sequence is unpickled (its __getstate__, sequence.py:98-106, does
    not send it), and count the last block's tokens from num_tokens (sequence.py:80-82
    slices token_ids, which a worker holds only in part during decode). On rank 0, whose
    token list is complete, both forms give the same number."""
    from myvllm.engine.sequence import Sequence
    if getattr(Sequence, "_mkv_worker_state", False):
        return
    unpickle = Sequence.__setstate__

    def setstate(self, state):
        unpickle(self, state)
        self.block_size = block_size

    Sequence.__setstate__ = setstate
    Sequence.last_block_num_tokens = property(
        lambda self: self.num_tokens - self.num_tokens // self.block_size * self.block_size)
    Sequence._mkv_worker_state = True


def install(impl: str, block_size: int) -> None:
    """The import-time changes listed in the module docstring (every rank)."""
    torch.set_default_dtype(torch.bfloat16)
    sequence_state_for_workers(block_size)
    # The reference's rotary cache is float32 (rotary_embedding.py:89), so a bf16 model's
    # q/k come out of RoPE as float32 and the float32 attention output then meets the
    # bf16 o_proj weight: the unmodified engine runs end to end only in float32. Cast
    # RoPE's outputs back to the input dtype (both arms alike).
    import myvllm.layers.rotary_embedding as rope
    rope_forward = rope.RotaryEmbedding.forward

    def rope_same_dtype(self, positions, query, key):
        q, k = rope_forward(self, positions, query, key)
        return q.to(query.dtype), k.to(key.dtype)

    rope.RotaryEmbedding.forward = rope_same_dtype
    import myvllm.utils.loader as loader
    loader.load_weights_from_checkpoint = random_weights
    if impl == "ours":
        import myvllm.models.qwen3 as q3
        import myvllm.utils.context as rctx
        ours = importlib.import_module(PKG + ".layers.attention")
        importlib.import_module(PKG).load()  # libmkv.so, loudly, before any model code
        ours.get_context = rctx.get_context  # the runner sets the reference's context
        q3.Attention = ours.Attention


def _worker(config: dict, rank: int, event, impl: str) -> None:
    install(impl, config["block_size"])
    from myvllm.engine.model_runner import ModelRunner
    runner = ModelRunner(config, rank, event)
    runner.loop()


def _patch_rendezvous(port: int) -> None:
    """The runner rendezvous at tcp://localhost:12345 (model_runner.py:28); give it a
    free port and 127.0.0.1 instead, so that two runs do not collide."""
    import torch.distributed as dist
    orig = dist.init_process_group

    def init(backend, init_method=None, *a, **kw):
        if isinstance(init_method, str) and init_method.startswith("tcp://localhost:"):
            init_method = f"tcp://127.0.0.1:{port}"
        return orig(backend, init_method, *a, **kw)

    dist.init_process_group = init


def _worker_entry(config, rank, event, impl):
    _patch_rendezvous(config["bench_port"])
    _worker(config, rank, event, impl)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--kv", default=None, help="kv_cache_dtype (default fp8_per_tensor for ours, auto for the reference)")
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--prompt-min", type=int, default=128)
    ap.add_argument("--prompt-max", type=int, default=1024)
    ap.add_argument("--output", type=int, default=256)
    ap.add_argument("--batched-tokens", type=int, default=8192)
    ap.add_argument("--max-seqs", type=int, default=256)
    ap.add_argument("--port", type=int, default=29571)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    kv = args.kv or ("fp8_per_tensor" if args.impl == "ours" else "auto")
    if not os.path.isdir(os.path.join(REF_DIR, "myvllm")):
        print(json.dumps({"impl": args.impl, "unavailable": "reference not installed in baseline/_ref"}))
        return
    if torch.cuda.device_count() < args.tp:
        print(json.dumps({"impl": args.impl, "unavailable": f"--tp {args.tp} needs {args.tp} GPUs"}))
        return

    import torch.multiprocessing as mp
    max_len = args.prompt_max + args.output
    config = qwen3_0p6b_config(args.tp, kv, max_len, args.batched_tokens, args.max_seqs, args.port)
    _patch_rendezvous(args.port)
    install(args.impl, config["block_size"])
    from myvllm.engine.model_runner import ModelRunner
    from myvllm.engine.scheduler import Scheduler
    from myvllm.engine.sequence import Sequence
    from myvllm.sampling_parameters import SamplingParams

    ctx = mp.get_context("spawn")
    events, procs = [], []
    for r in range(1, args.tp):
        ev = ctx.Event()
        pr = ctx.Process(target=_worker_entry, args=(config, r, ev, args.impl))
        pr.start()
        events.append(ev)
        procs.append(pr)
    t_init = time.perf_counter()
    runner = ModelRunner(config, 0, events)
    init_s = time.perf_counter() - t_init
    scheduler = Scheduler(max_num_sequences=config["max_num_sequences"],
                          max_num_batched_tokens=config["max_num_batched_tokens"],
                          max_cached_blocks=config["max_cached_blocks"],
                          block_size=config["block_size"], eos=config["eos"],
                          enable_chunked_prefill=True)

    gen = torch.Generator().manual_seed(args.seed)
    params = SamplingParams(temperature=0.6, max_tokens=args.output, ignore_eos=True,
                            max_model_length=max_len)

    def add(n_req, n_out=None):
        p = params if n_out is None else SamplingParams(temperature=0.6, max_tokens=n_out,
                                                        ignore_eos=True, max_model_length=max_len)
        lens = torch.randint(args.prompt_min, args.prompt_max + 1, (n_req,), generator=gen,
                             device="cpu").tolist()
        for n in lens:
            ids = torch.randint(0, config["vocab_size"], (n,), generator=gen, device="cpu").tolist()
            scheduler.add_sequence(Sequence(token_ids=ids, block_size=config["block_size"],
                                            sampling_params=p))
        return sum(lens)

    def run_all():
        """Engine steps until every sequence is finished (llm_engine.py:76-92)."""
        out_tokens = dec_tokens = dec_steps = steps = 0
        dec_time = 0.0
        t0 = time.perf_counter()
        while not scheduler.is_finished():
            ts = time.perf_counter()
            items, is_prefill = scheduler.schedule()
            if not items:
                continue
            # the runner's own test for a decode-only batch (model_runner.py:720-722)
            decode_only = all(it.seq.num_computed_tokens >= it.seq.num_prompt_tokens for it in items)
            outputs = runner.call("run", items, is_prefill)
            outputs = outputs.cpu().tolist() if outputs is not None else []
            scheduler.postprocess(items, outputs)
            dt = time.perf_counter() - ts
            steps += 1
            out_tokens += len(outputs)
            if decode_only:
                dec_steps += 1
                dec_tokens += len(outputs)
                dec_time += dt
        torch.cuda.synchronize()
        return time.perf_counter() - t0, out_tokens, steps, dec_tokens, dec_steps, dec_time

    add(min(16, args.requests), 8)  # warm-up: kernels compiled / loaded, FP8 scales calibrated
    run_all()
    prompt_tokens = add(args.requests)
    wall, out_tokens, steps, dec_tokens, dec_steps, dec_time = run_all()
    line = {
        "metric": "decode tokens/s (BASELINE config 5, reference engine)", "impl": args.impl,
        "tp": args.tp, "kv_cache_dtype": kv, "dtype": "bf16",
        "data": "synthetic (random token ids, random-init weights)",
        "config": {"model": "Qwen3-0.6B shape (random init)", "requests": args.requests,
                   "prompt_len": [args.prompt_min, args.prompt_max], "output_tokens": args.output,
                   "temperature": 0.6, "ignore_eos": True, "chunked_prefill": True,
                   "max_num_batched_tokens": args.batched_tokens, "max_num_sequences": args.max_seqs,
                   "enforce_eager": True, "attention": "libmkv" if args.impl == "ours" else "reference Triton"},
        "prompt_tokens": prompt_tokens, "generated_tokens": out_tokens, "wall_s": round(wall, 3),
        "tokens_per_s": round(out_tokens / wall, 1),
        "decode_steps": dec_steps, "decode_tokens_per_s": round(dec_tokens / dec_time, 1) if dec_time else None,
        "engine_steps": steps, "init_s": round(init_s, 1),
    }
    runner.call("exit")
    for pr in procs:
        pr.join(timeout=120)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
