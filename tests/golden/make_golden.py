"""Generates tests/golden/*.npz by running the reference's own code on seeded inputs.

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --reference-src DIR

DIR is the `src` directory of a checkout of the reference (heart1128/mini-kvllm), or
MKV_REFERENCE_SRC when the option is not given; its parent must hold
benchmark_decoding.py. The script needs
the reference only while it runs: the fixtures it writes carry the inputs (or the
seed and a SHA-256 of them) and the reference's outputs, and the tests read only
those files.

What runs, per fixture (all on the CPU):
  append_bf16      store_kvcache (attention.py:67), Triton kernel interpreted
  append_fp8       store_kvcache_fp8 (attention.py:281), per-tensor mode, twice
                   (calibration on the first call, frozen scale on the second). The
                   Triton interpreter's fp32->e4m3 cast is known to be wrong for values
                   that round up into the next binade, so the kernel is run with float32
                   "caches": it then stores clamp(x / scale, -448, 448) as fp32, and the
                   fixture keeps those values plus the scales the reference calibrated.
  decode_small     paged_attention_decode (attention.py:895), interpreted, fp32, with
                   ragged lengths, -1 padding and a -1 page inside one context
  decode_fp8       paged_attention_decode_quantized(..., 'fp8_per_tensor')
                   (attention.py:1213) on e4m3-representable values held in fp32 caches
  decode_config1   decode_torch_optimized (benchmark_decoding.py:145-198, loaded from
                   the file's source text because the module's imports are stale) on
                   B=4, H=16, KVH=8, D=128, BS=16, ctx ~ U[64, 512]
  append_fp8_pth   store_kvcache_fp8(..., 'fp8_per_token_head') (attention.py:118-191,
                   PER_TOKEN_HEAD=1) on float32 "caches": per-(slot, head) scales and
                   pre-cast quotients
  append_int8      store_kvcache_int8 (attention.py:195-278): int8 bytes and scales
  decode_fp8_pth,  paged_attention_decode_quantized with 'fp8_per_token_head' /
  decode_int8      'int8_per_token_head' (the tile kernel, attention.py:1124-1210)
  prefill          paged_attention_prefill_triton (attention.py:852-892; kernel 704-849),
                   chunked prefill over cached prefixes with a -1 page inside one context
  varlen_prefill   flash_attention_prefill (attention.py:446-516; kernel 336-443), causal
                   attention of ragged sequences over their own contiguous K/V, fp32
  residual_rmsnorm LayerNorm.residual_rms_forward (layernorm.py:25-27) after a summed
                   all-reduce (linear.py:222-225), run eagerly (see the function)
"""
from __future__ import annotations

import argparse
import ast
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference(src: str):
    os.environ.setdefault("TRITON_INTERPRET", "1")
    sys.path.insert(0, src)
    import torch  # noqa: F401
    from myvllm.layers import attention as ref_attn  # the reference module itself

    bench_path = os.path.join(os.path.dirname(src), "benchmark_decoding.py")
    text = open(bench_path).read()
    tree = ast.parse(text)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "decode_torch_optimized")
    mod = ast.Module(body=[fn], type_ignores=[])
    ns: dict = {"torch": __import__("torch")}
    exec(compile(mod, bench_path, "exec"), ns)
    return ref_attn, ns["decode_torch_optimized"]


def _sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _bf16_bits(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().astype(np.uint16)


def make_append_bf16(ref_attn, rng):
    import torch
    T, KVH, D, NB, BS = 37, 2, 32, 12, 4
    key = torch.from_numpy(rng.standard_normal((T, KVH, D)).astype(np.float32)).to(torch.bfloat16)
    value = torch.from_numpy(rng.standard_normal((T, KVH, D)).astype(np.float32)).to(torch.bfloat16)
    slots = torch.from_numpy(rng.permutation(NB * BS)[:T].astype(np.int64))
    slots[[3, 10, 11, 30]] = -1
    kc0 = torch.from_numpy(rng.standard_normal((NB, BS, KVH, D)).astype(np.float32)).to(torch.bfloat16)
    vc0 = torch.from_numpy(rng.standard_normal((NB, BS, KVH, D)).astype(np.float32)).to(torch.bfloat16)
    kc, vc = kc0.clone(), vc0.clone()
    ref_attn.store_kvcache(key, value, kc, vc, slots, BS)
    return dict(key=_bf16_bits(key), value=_bf16_bits(value), slot_mapping=slots.numpy(),
                k_cache_in=_bf16_bits(kc0), v_cache_in=_bf16_bits(vc0),
                k_cache_out=_bf16_bits(kc), v_cache_out=_bf16_bits(vc),
                block_size=np.int64(BS))


def make_append_fp8(ref_attn, rng):
    import torch
    T, KVH, D, NB, BS = 24, 2, 32, 8, 4
    out = {}
    kc = torch.zeros(NB, BS, KVH, D, dtype=torch.float32)
    vc = torch.zeros(NB, BS, KVH, D, dtype=torch.float32)
    k_scale = torch.ones(1, dtype=torch.float32)
    v_scale = torch.ones(1, dtype=torch.float32)
    perm = rng.permutation(NB * BS)
    for call in range(2):
        x = rng.standard_normal((2, T, KVH, D)).astype(np.float32)
        mask = rng.random((2, T, KVH, D)) < 0.01
        x = np.where(mask, x * 20.0, x)  # 0.1%-1% outliers x20
        key = torch.from_numpy(x[0]).to(torch.bfloat16)
        value = torch.from_numpy(x[1]).to(torch.bfloat16)
        # second call: 24 slots overlapping the first call's last 16 (overwrites)
        lo = 0 if call == 0 else NB * BS - T
        slots = torch.from_numpy(perm[lo:lo + T].astype(np.int64))
        slots[[1, 7]] = -1
        ref_attn.store_kvcache_fp8(key, value, kc, vc, k_scale, v_scale, slots, BS, "fp8_per_tensor")
        out[f"key{call}"] = _bf16_bits(key)
        out[f"value{call}"] = _bf16_bits(value)
        out[f"slot_mapping{call}"] = slots.numpy()
        out[f"k_scale{call}"] = k_scale.numpy().copy()
        out[f"v_scale{call}"] = v_scale.numpy().copy()
        out[f"k_quot{call}"] = kc.numpy().copy()  # clamp(x/scale) as fp32, before the e4m3 cast
        out[f"v_quot{call}"] = vc.numpy().copy()
    out["block_size"] = np.int64(BS)
    return out


def _pth_rows(rng, T, KVH, D):
    """bf16 K/V rows with 1% outliers x20, plus an all-zero row and a row of ties."""
    import torch
    x = rng.standard_normal((2, T, KVH, D)).astype(np.float32)
    x = np.where(rng.random((2, T, KVH, D)) < 0.01, x * 20.0, x)
    x[:, 5, 1, :] = 0.0                      # amax 0: FP8 scale 1.0, INT8 scale 1e-6
    x[:, 9, 0, :] = np.tile([2.5, -2.5, 0.5, -127.0], D // 4)  # exact halves after scaling
    return torch.from_numpy(x[0]).to(torch.bfloat16), torch.from_numpy(x[1]).to(torch.bfloat16)


def make_append_pth(ref_attn, rng, mode):
    """store_kvcache_fp8(..., 'fp8_per_token_head') or store_kvcache_int8 on 24 tokens.
    FP8 runs with float32 "caches" (see append_fp8) and keeps the pre-cast quotients;
    INT8 writes int8 caches directly (the interpreter's float->int8 conversion truncates
    toward zero, as the GPU's does)."""
    import torch
    T, KVH, D, NB, BS = 24, 2, 32, 8, 4
    key, value = _pth_rows(rng, T, KVH, D)
    slots = torch.from_numpy(rng.permutation(NB * BS)[:T].astype(np.int64))
    slots[[1, 7]] = -1
    ks = torch.full((NB, BS, KVH), -1.0, dtype=torch.float32)  # -1 marks slots not written
    vs = torch.full((NB, BS, KVH), -1.0, dtype=torch.float32)
    if mode == "fp8":
        kc = torch.zeros(NB, BS, KVH, D, dtype=torch.float32)
        vc = torch.zeros(NB, BS, KVH, D, dtype=torch.float32)
        ref_attn.store_kvcache_fp8(key, value, kc, vc, ks, vs, slots, BS, "fp8_per_token_head")
        caches = dict(k_quot=kc.numpy(), v_quot=vc.numpy())
    else:
        kc = torch.zeros(NB, BS, KVH, D, dtype=torch.int8)
        vc = torch.zeros(NB, BS, KVH, D, dtype=torch.int8)
        ref_attn.store_kvcache_int8(key, value, kc, vc, ks, vs, slots, BS)
        caches = dict(k_cache=kc.numpy(), v_cache=vc.numpy())
    return dict(key=_bf16_bits(key), value=_bf16_bits(value), slot_mapping=slots.numpy(),
                k_scales=ks.numpy(), v_scales=vs.numpy(), block_size=np.int64(BS), **caches)


def make_decode_pth(ref_attn, rng, mode):
    """paged_attention_decode_quantized(..., 'fp8_per_token_head' | 'int8_per_token_head')
    with head_dim <= 128, i.e. the reference's tile kernel (attention.py:1124-1210): FP8
    codes held in float32 caches (the kernel converts loads to float32 either way), INT8
    caches as int8, per-(page, row, kv head) scales. No -1 page lies inside a context
    (that kernel would give such tokens score 0 rather than skip them)."""
    import torch
    B, H, KVH, D, BS, MAXB = 4, 8, 2, 32, 8, 6
    lens = [5, 48, 20, 33]
    q, kc, vc, bt, cl = _paged_inputs(rng, B, H, KVH, D, BS, lens, MAXB)
    NB = kc.shape[0]
    ks = (rng.random((NB, BS, KVH)) * 0.04 + 0.005).astype(np.float32)
    vs = (rng.random((NB, BS, KVH)) * 0.04 + 0.005).astype(np.float32)
    if mode == "fp8":
        k = torch.from_numpy(kc * 40).to(torch.float8_e4m3fn)
        v = torch.from_numpy(vc * 40).to(torch.float8_e4m3fn)
        kin, vin = k.float(), v.float()
        codes = dict(k_cache_e4m3=k.view(torch.uint8).numpy(), v_cache_e4m3=v.view(torch.uint8).numpy())
        kvd = "fp8_per_token_head"
    else:
        kin = torch.from_numpy(np.clip(np.rint(kc * 40), -128, 127).astype(np.int8))
        vin = torch.from_numpy(np.clip(np.rint(vc * 40), -128, 127).astype(np.int8))
        codes = dict(k_cache_i8=kin.numpy(), v_cache_i8=vin.numpy())
        kvd = "int8_per_token_head"
    scale = 1.0 / np.sqrt(D)
    out = ref_attn.paged_attention_decode_quantized(
        torch.from_numpy(q), kin, vin, torch.from_numpy(ks), torch.from_numpy(vs),
        torch.from_numpy(bt), torch.from_numpy(cl), float(scale), H, KVH, D, BS, kvd)
    return dict(query=q, k_scales=ks, v_scales=vs, block_tables=bt, context_lens=cl,
                scale=np.float64(scale), num_heads=np.int64(H), num_kv_heads=np.int64(KVH),
                block_size=np.int64(BS), out=out.numpy(), **codes)


def make_prefill(ref_attn, rng):
    """paged_attention_prefill_triton (attention.py:852-892) and paged_attention_prefill_torch
    (649-701), interpreted: 3 sequences extending a cached prefix (chunked prefill), one
    starting at position 0, one chunk of a single token, and a -1 page inside a context;
    fp32 pages."""
    import torch
    B, H, KVH, D, BS, MAXB = 3, 4, 2, 32, 4, 9
    ctx = [13, 30, 7]                  # tokens in the cache after this chunk was appended
    chunk = [5, 1, 7]                  # new query tokens per sequence (the last ctx tokens)
    q_, kc, vc, bt, cl = _paged_inputs(rng, B, H, KVH, D, BS, ctx, MAXB)
    bt[1, 2] = -1                      # a -1 page inside sequence 1's context
    cu = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    pos = np.concatenate([np.arange(c - n, c) for c, n in zip(ctx, chunk)]).astype(np.int64)
    q = rng.standard_normal((int(cu[-1]), H, D)).astype(np.float32)
    scale = 1.0 / np.sqrt(D)
    args = (torch.from_numpy(q), torch.from_numpy(kc), torch.from_numpy(vc), torch.from_numpy(bt),
            torch.from_numpy(cl), torch.from_numpy(cu), torch.from_numpy(pos), float(scale))
    out_triton = ref_attn.paged_attention_prefill_triton(*args, H, KVH, D, BS)
    # paged_attention_prefill_torch indexes every page it reads (a -1 entry would read the
    # last block through Python's negative indexing), so it runs on the same inputs with
    # the -1 entry replaced by the page the triton case skipped
    bt_t = bt.copy()
    bt_t[1, 2] = int(bt[1, 3]) if bt[1, 3] >= 0 else 0
    out_torch = ref_attn.paged_attention_prefill_torch(
        torch.from_numpy(q), torch.from_numpy(kc), torch.from_numpy(vc), torch.from_numpy(bt_t),
        torch.from_numpy(cl), torch.from_numpy(cu), torch.from_numpy(pos), float(scale), H, KVH, BS)
    return dict(query=q, k_cache=kc, v_cache=vc, block_tables=bt, context_lens=cl, cu_seqlens_q=cu,
                positions=pos, scale=np.float64(scale), num_heads=np.int64(H),
                num_kv_heads=np.int64(KVH), block_size=np.int64(BS), out=out_triton.numpy(),
                block_tables_torch=bt_t, out_torch=out_torch.numpy())


def _paged_inputs(rng, B, H, KVH, D, BS, lens, max_blocks, extra_blocks=3):
    import torch
    need = [(n + BS - 1) // BS for n in lens]
    NB = sum(need) + extra_blocks
    perm = rng.permutation(NB)
    bt = np.full((B, max_blocks), -1, dtype=np.int32)
    pos = 0
    for b, nb in enumerate(need):
        nb_in = min(nb, max_blocks)
        bt[b, :nb_in] = perm[pos:pos + nb_in]
        pos += nb
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    kc = rng.standard_normal((NB, BS, KVH, D)).astype(np.float32)
    vc = rng.standard_normal((NB, BS, KVH, D)).astype(np.float32)
    return q, kc, vc, bt, np.asarray(lens, dtype=np.int64)


def make_decode_small(ref_attn, rng):
    import torch
    B, H, KVH, D, BS, MAXB = 8, 4, 2, 32, 4, 10
    # 40 = MAXB*BS; 4 = one full block; 45 > MAXB*BS (tokens 40..44 have no table
    # entry and are dropped); 0 = no visible token (the reference returns 0/0 = NaN)
    lens = [1, 4, 17, 40, 9, 23, 45, 0]
    q, kc, vc, bt, cl = _paged_inputs(rng, B, H, KVH, D, BS, lens, MAXB)
    bt[4, 1] = -1  # a -1 page inside a context: its 4 tokens carry no weight
    scale = 1.0 / np.sqrt(D)
    out = ref_attn.paged_attention_decode(
        torch.from_numpy(q), torch.from_numpy(kc), torch.from_numpy(vc), torch.from_numpy(bt),
        torch.from_numpy(cl), float(scale), H, KVH, D, BS)
    return dict(query=q, k_cache=kc, v_cache=vc, block_tables=bt, context_lens=cl,
                scale=np.float64(scale), num_heads=np.int64(H), num_kv_heads=np.int64(KVH),
                block_size=np.int64(BS), out=out.numpy())


def make_decode_fp8(ref_attn, rng):
    import torch
    B, H, KVH, D, BS, MAXB = 4, 8, 2, 32, 8, 6
    lens = [5, 48, 20, 33]
    q, kc, vc, bt, cl = _paged_inputs(rng, B, H, KVH, D, BS, lens, MAXB)
    k8 = torch.from_numpy(kc * 40).to(torch.float8_e4m3fn)  # e4m3 codes
    v8 = torch.from_numpy(vc * 40).to(torch.float8_e4m3fn)
    ks = torch.tensor([0.0213623046875], dtype=torch.float32)
    vs = torch.tensor([0.031982421875], dtype=torch.float32)
    scale = 1.0 / np.sqrt(D)
    out = ref_attn.paged_attention_decode_quantized(
        torch.from_numpy(q), k8.float(), v8.float(), ks, vs, torch.from_numpy(bt),
        torch.from_numpy(cl), float(scale), H, KVH, D, BS, "fp8_per_tensor")
    return dict(query=q, k_cache_e4m3=k8.view(torch.uint8).numpy(),
                v_cache_e4m3=v8.view(torch.uint8).numpy(), k_scale=ks.numpy(), v_scale=vs.numpy(),
                block_tables=bt, context_lens=cl, scale=np.float64(scale), num_heads=np.int64(H),
                num_kv_heads=np.int64(KVH), block_size=np.int64(BS), out=out.numpy())


def config1_inputs(seed: int = 0):
    """BASELINE config 1 (shared with tests): B=4, H=16, KVH=8, D=128, BS=16,
    ctx ~ U[64, 512], pages a random permutation, q/K/V ~ N(0, 1) fp32."""
    rng = np.random.default_rng(seed)
    B, H, KVH, D, BS, MAXB = 4, 16, 8, 128, 16, 32
    lens = rng.integers(64, 513, size=B).tolist()
    q, kc, vc, bt, cl = _paged_inputs(rng, B, H, KVH, D, BS, lens, MAXB, extra_blocks=0)
    return dict(query=q, k_cache=kc, v_cache=vc, block_tables=bt, context_lens=cl,
                num_heads=H, num_kv_heads=KVH, head_dim=D, block_size=BS)


def make_decode_config1(decode_torch_optimized):
    import torch
    inp = config1_inputs(0)
    D = inp["head_dim"]
    scale = 1.0 / np.sqrt(D)
    out = decode_torch_optimized(
        torch.from_numpy(inp["query"]), torch.from_numpy(inp["k_cache"]),
        torch.from_numpy(inp["v_cache"]), torch.from_numpy(inp["block_tables"]),
        torch.from_numpy(inp["context_lens"]), float(scale), inp["num_heads"],
        inp["num_kv_heads"], D, inp["block_size"])
    digest = _sha(inp["query"], inp["k_cache"], inp["v_cache"], inp["block_tables"], inp["context_lens"])
    return dict(seed=np.int64(0), inputs_sha256=np.array(digest), scale=np.float64(scale),
                context_lens=inp["context_lens"], out=out.numpy())


def make_residual_rmsnorm(src, rng):
    """LayerNorm.residual_rms_forward (layernorm.py:25-27) of the reference, the op that
    follows RowParallelLinear's all-reduce (linear.py:222-225). Its rms_forward is wrapped
    in torch.compile, whose CPU backend needs OpenMP (absent here), so it runs eagerly
    (dynamo disabled): s = x + residual is a bf16 add either way; the normalisation is
    computed in bf16 steps here and in fp32 by the compiled GPU code, so `out` pins the
    formula to bf16 accuracy. x is the bf16 rounding of the fp32 sum of four partials."""
    import torch
    import torch._dynamo
    torch._dynamo.config.disable = True
    sys.path.insert(0, src)
    from myvllm.layers.layernorm import LayerNorm
    T, H, N = 8, 1024, 4
    partials = torch.from_numpy(rng.standard_normal((N, T, H)).astype(np.float32)).bfloat16()
    residual = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32) * 2).bfloat16()
    weight = torch.from_numpy(rng.uniform(0.5, 1.5, H).astype(np.float32)).bfloat16()
    x = partials.float().sum(0).bfloat16()
    ln = LayerNorm(weight, eps=1e-6)
    with torch.no_grad():
        out, s = ln(x, residual)
    return dict(partials=_bf16_bits(partials), residual=_bf16_bits(residual), weight=_bf16_bits(weight),
                eps=np.float64(1e-6), x=_bf16_bits(x), s=_bf16_bits(s), out=_bf16_bits(out))


def make_varlen_prefill(ref_attn, rng):
    import torch
    H, KVH, D = 4, 2, 32
    lens = [5, 37, 1, 64, 70]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    q = rng.standard_normal((T, H, D)).astype(np.float32)
    k = rng.standard_normal((T, KVH, D)).astype(np.float32)
    v = rng.standard_normal((T, KVH, D)).astype(np.float32)
    scale = 1.0 / np.sqrt(D)
    out = ref_attn.flash_attention_prefill(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
                                           torch.from_numpy(cu), float(scale), H, KVH, D)
    return dict(query=q, key=k, value=v, cu_seqlens=cu, scale=np.float64(scale),
                num_heads=np.int64(H), num_kv_heads=np.int64(KVH), out=out.numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("MKV_REFERENCE_SRC"),
                    required="MKV_REFERENCE_SRC" not in os.environ)
    ap.add_argument("--only", default="", help="comma-separated fixture names")
    args = ap.parse_args()
    ref_attn, dto = _load_reference(args.reference_src)
    jobs = [
        ("append_bf16", lambda: make_append_bf16(ref_attn, np.random.default_rng(101))),
        ("append_fp8", lambda: make_append_fp8(ref_attn, np.random.default_rng(202))),
        ("decode_small", lambda: make_decode_small(ref_attn, np.random.default_rng(303))),
        ("decode_fp8", lambda: make_decode_fp8(ref_attn, np.random.default_rng(404))),
        ("decode_config1", lambda: make_decode_config1(dto)),
        ("append_fp8_pth", lambda: make_append_pth(ref_attn, np.random.default_rng(505), "fp8")),
        ("append_int8", lambda: make_append_pth(ref_attn, np.random.default_rng(606), "int8")),
        ("decode_fp8_pth", lambda: make_decode_pth(ref_attn, np.random.default_rng(707), "fp8")),
        ("decode_int8", lambda: make_decode_pth(ref_attn, np.random.default_rng(808), "int8")),
        ("prefill", lambda: make_prefill(ref_attn, np.random.default_rng(909))),
        ("residual_rmsnorm", lambda: make_residual_rmsnorm(args.reference_src, np.random.default_rng(1010))),
        ("varlen_prefill", lambda: make_varlen_prefill(ref_attn, np.random.default_rng(1111))),
    ]
    only = set(args.only.split(",")) if args.only else None
    for name, job in jobs:
        if only and name not in only:
            continue
        data = job()
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **data)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
