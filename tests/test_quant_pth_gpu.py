"""KV caches quantised per (token, kv head): FP8 E4M3 ('fp8_per_token_head') and INT8
('int8_per_token_head') appends and decodes on the GPU through the public wrappers,
against the CPU oracle (restated from attention.py:118-278 and 1124-1268, pinned by
tests/golden/{append_fp8_pth,append_int8,decode_fp8_pth,decode_int8}.npz).

Append: bytes and scales bit-exact. Decode: atol 2e-2 / rtol 1e-2 for bf16/fp16
queries (fp32 accumulation over f16 tensor-core operands), atol 2e-5 / rtol 1e-4 for
fp32 queries."""
import math

import numpy as np
import pytest
import torch

from conftest import golden, mkv_module
from oracle import paged_decode_ref, store_kvcache_quant_per_token_head_ref

pytestmark = pytest.mark.gpu
attn = mkv_module("layers.attention")

TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (2e-2, 1e-2), torch.bfloat16: (2e-2, 1e-2)}
CACHE = {"fp8": torch.float8_e4m3fn, "int8": torch.int8}
MODE = {"fp8": "fp8_per_token_head", "int8": "int8_per_token_head"}


def bf16(a):
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)


def _store_cuda(mode, key, value, kc, vc, ks, vs, slots, bs):
    k, v, kc, vc, ks, vs, sl = (t.cuda() for t in (key, value, kc, vc, ks, vs, slots))
    if mode == "int8":
        attn.store_kvcache_int8(k, v, kc, vc, ks, vs, sl, bs)
    else:
        attn.store_kvcache_fp8(k, v, kc, vc, ks, vs, sl, bs, "fp8_per_token_head")
    return kc.cpu(), vc.cpu(), ks.cpu(), vs.cpu()


def _rows(T, KVH, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2, T, KVH, D, generator=g)
    x = torch.where(torch.rand(2, T, KVH, D, generator=g) < 0.001, x * 20.0, x)  # config 2 outliers
    x[:, 3 % T, 0, :] = 0.0  # all-zero row
    return x[0].to(dtype), x[1].to(dtype)


@pytest.mark.parametrize("mode", ["fp8", "int8"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [128, 64, 96, 256])
def test_append_per_token_head_bit_exact(mode, dtype, D):
    T, KVH, BS, NB = 300, 8, 256, 4
    key, value = _rows(T, KVH, D, dtype, seed=D + 7)
    g = torch.Generator().manual_seed(11)
    slots = torch.randperm(NB * BS, generator=g)[:T].long()
    slots[[1, 50, 299]] = -1
    shape = (NB, BS, KVH, D)
    kc0 = torch.zeros(shape, dtype=CACHE[mode])
    ks0 = torch.full((NB, BS, KVH), -1.0)
    ref = [kc0.clone(), kc0.clone(), ks0.clone(), ks0.clone()]
    store_kvcache_quant_per_token_head_ref(key, value, *ref, slots, BS, mode)
    got = _store_cuda(mode, key, value, kc0.clone(), kc0.clone(), ks0.clone(), ks0.clone(), slots, BS)
    for a, b in zip(got, ref):
        assert torch.equal(a.view(torch.uint8) if a.dtype != torch.float32 else a,
                           b.view(torch.uint8) if b.dtype != torch.float32 else b)


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_append_per_token_head_nan_rows(mode):
    """A row holding NaN: scale 1 (FP8) / 1e-6 (INT8); NaN elements store -448 / -128,
    the others are quantised with that scale (saturating for INT8)."""
    T, KVH, D, BS, NB = 8, 2, 128, 16, 2
    key, value = _rows(T, KVH, D, torch.bfloat16, seed=5)
    key[2, 1, 7] = float("nan")
    value[6, 0, 0] = float("nan")
    slots = torch.arange(T, dtype=torch.int64)
    shape = (NB, BS, KVH, D)
    ref = [torch.zeros(shape, dtype=CACHE[mode]), torch.zeros(shape, dtype=CACHE[mode]),
           torch.zeros(NB, BS, KVH), torch.zeros(NB, BS, KVH)]
    store_kvcache_quant_per_token_head_ref(key, value, *ref, slots, BS, mode)
    got = _store_cuda(mode, key, value, torch.zeros(shape, dtype=CACHE[mode]),
                      torch.zeros(shape, dtype=CACHE[mode]), torch.zeros(NB, BS, KVH),
                      torch.zeros(NB, BS, KVH), slots, BS)
    assert float(got[2][0, 2, 1]) == (1.0 if mode == "fp8" else float(np.float32(1e-6)))
    for a, b in zip(got, ref):
        assert torch.equal(a.view(torch.uint8) if a.dtype != torch.float32 else a,
                           b.view(torch.uint8) if b.dtype != torch.float32 else b)


def test_golden_int8_append_through_cuda():
    g = golden("append_int8")
    shape = g["k_cache"].shape
    got = _store_cuda("int8", bf16(g["key"]), bf16(g["value"]), torch.zeros(shape, dtype=torch.int8),
                      torch.zeros(shape, dtype=torch.int8), torch.full(g["k_scales"].shape, -1.0),
                      torch.full(g["v_scales"].shape, -1.0), torch.from_numpy(g["slot_mapping"]),
                      int(g["block_size"]))
    assert torch.equal(got[0], torch.from_numpy(g["k_cache"]))
    assert torch.equal(got[1], torch.from_numpy(g["v_cache"]))
    assert torch.equal(got[2], torch.from_numpy(g["k_scales"]))
    assert torch.equal(got[3], torch.from_numpy(g["v_scales"]))


def test_golden_fp8_per_token_head_append_through_cuda():
    g = golden("append_fp8_pth")
    shape = g["k_quot"].shape
    got = _store_cuda("fp8", bf16(g["key"]), bf16(g["value"]),
                      torch.zeros(shape, dtype=torch.float8_e4m3fn),
                      torch.zeros(shape, dtype=torch.float8_e4m3fn),
                      torch.full(g["k_scales"].shape, -1.0), torch.full(g["v_scales"].shape, -1.0),
                      torch.from_numpy(g["slot_mapping"]), int(g["block_size"]))
    assert torch.equal(got[2], torch.from_numpy(g["k_scales"]))
    assert torch.equal(got[3], torch.from_numpy(g["v_scales"]))
    exp_k = torch.from_numpy(g["k_quot"]).to(torch.float8_e4m3fn)
    exp_v = torch.from_numpy(g["v_quot"]).to(torch.float8_e4m3fn)
    assert torch.equal(got[0].view(torch.uint8), exp_k.view(torch.uint8))
    assert torch.equal(got[1].view(torch.uint8), exp_v.view(torch.uint8))


# ------------------------------------------------------------------------------ decode
def _paged(B, H, KVH, D, BS, lens, mode, seed, qdtype):
    g = torch.Generator().manual_seed(seed)
    need = [(n + BS - 1) // BS for n in lens]
    NB = sum(need) + 3
    perm = torch.randperm(NB, generator=g)
    bt = torch.full((B, max(max(need), 1)), -1, dtype=torch.int32)
    pos = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[pos:pos + k].int()
        pos += k
    q = torch.randn(B, H, D, generator=g).to(qdtype)
    raw = torch.randn(2, NB, BS, KVH, D, generator=g) * 40
    if mode == "fp8":
        kc, vc = raw[0].to(torch.float8_e4m3fn), raw[1].to(torch.float8_e4m3fn)
    else:
        kc, vc = raw[0].round().clamp(-128, 127).to(torch.int8), raw[1].round().clamp(-128, 127).to(torch.int8)
    ks = torch.rand(NB, BS, KVH, generator=g) * 0.04 + 0.002
    vs = torch.rand(NB, BS, KVH, generator=g) * 0.04 + 0.002
    return q, kc, vc, ks, vs, bt, torch.tensor(lens, dtype=torch.int64)


def _decode_cuda(mode, q, kc, vc, ks, vs, bt, cl, scale, H, KVH, D, BS, splits=0):
    return attn.paged_attention_decode_quantized(
        q.cuda(), kc.cuda(), vc.cuda(), ks.cuda(), vs.cuda(), bt.cuda(), cl.cuda(), scale, H, KVH, D,
        BS, MODE[mode], num_splits=splits).cpu()


def _close(out, ref, dtype):
    atol, rtol = TOL[dtype]
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(out), nan), "NaN pattern differs"
    diff = (out.double() - ref)[~nan].abs()
    assert bool((diff <= atol + rtol * ref[~nan].abs()).all()), f"max abs err {float(diff.max()):.3e}"


LENS = [1, 16, 17, 63, 64, 65, 200, 511, 0, 300, 1500]


@pytest.mark.parametrize("mode", ["fp8", "int8"])
@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("H,KVH", [(32, 8), (8, 8), (32, 2)])
@pytest.mark.parametrize("BS", [16, 256])
def test_decode_per_token_head_matches_oracle(mode, qdtype, H, KVH, BS):
    D = 128
    q, kc, vc, ks, vs, bt, cl = _paged(len(LENS), H, KVH, D, BS, LENS, mode, seed=H + KVH + BS, qdtype=qdtype)
    scale = 1.0 / math.sqrt(D)
    ref = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS, k_scales=ks, v_scales=vs)
    _close(_decode_cuda(mode, q, kc, vc, ks, vs, bt, cl, scale, H, KVH, D, BS), ref, qdtype)


@pytest.mark.parametrize("mode", ["fp8", "int8"])
@pytest.mark.parametrize("splits", [1, 3, 64])
def test_decode_per_token_head_forced_splits(mode, splits):
    H, KVH, D, BS = 32, 8, 128, 16
    lens = [1000, 1, 0, 777, 129]
    q, kc, vc, ks, vs, bt, cl = _paged(len(lens), H, KVH, D, BS, lens, mode, seed=splits, qdtype=torch.bfloat16)
    ref = paged_decode_ref(q, kc, vc, bt, cl, 0.088, H, KVH, D, BS, k_scales=ks, v_scales=vs)
    _close(_decode_cuda(mode, q, kc, vc, ks, vs, bt, cl, 0.088, H, KVH, D, BS, splits), ref, torch.bfloat16)


@pytest.mark.parametrize("mode", ["fp8", "int8"])
@pytest.mark.parametrize("D", [64, 256])
def test_decode_per_token_head_other_head_dims(mode, D):
    H, KVH, BS = 8, 2, 16
    q, kc, vc, ks, vs, bt, cl = _paged(len(LENS), H, KVH, D, BS, LENS, mode, seed=D, qdtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    ref = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS, k_scales=ks, v_scales=vs)
    _close(_decode_cuda(mode, q, kc, vc, ks, vs, bt, cl, scale, H, KVH, D, BS), ref, torch.bfloat16)


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_golden_per_token_head_decode_through_cuda(mode):
    g = golden("decode_fp8_pth" if mode == "fp8" else "decode_int8")
    H, KVH, BS = int(g["num_heads"]), int(g["num_kv_heads"]), int(g["block_size"])
    q = torch.from_numpy(g["query"])
    if mode == "fp8":
        kc = torch.from_numpy(g["k_cache_e4m3"]).view(torch.float8_e4m3fn)
        vc = torch.from_numpy(g["v_cache_e4m3"]).view(torch.float8_e4m3fn)
    else:
        kc, vc = torch.from_numpy(g["k_cache_i8"]), torch.from_numpy(g["v_cache_i8"])
    out = _decode_cuda(mode, q, kc, vc, torch.from_numpy(g["k_scales"]), torch.from_numpy(g["v_scales"]),
                       torch.from_numpy(g["block_tables"]), torch.from_numpy(g["context_lens"]),
                       float(g["scale"]), H, KVH, q.shape[2], BS)
    _close(out, torch.from_numpy(g["out"]).double(), torch.float32)


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_append_then_decode_round_trip(mode):
    """Quantise a batch of K/V into the pages with the append, then decode: equals the
    oracle's decode over the oracle's quantised pages and scales."""
    B, H, KVH, D, BS = 6, 16, 4, 128, 16
    lens = [90, 1, 33, 250, 16, 47]
    T = sum(lens)
    NB = sum((n + BS - 1) // BS for n in lens) + 2
    g = torch.Generator().manual_seed(21)
    perm = torch.randperm(NB, generator=g)
    bt = torch.full((B, max((n + BS - 1) // BS for n in lens)), -1, dtype=torch.int32)
    slots, pos = [], 0
    for b, n in enumerate(lens):
        k = (n + BS - 1) // BS
        bt[b, :k] = perm[pos:pos + k].int()
        pos += k
        slots += [int(bt[b, t // BS]) * BS + t % BS for t in range(n)]
    slots = torch.tensor(slots, dtype=torch.int64)
    key, value = _rows(T, KVH, D, torch.bfloat16, seed=22)
    shape = (NB, BS, KVH, D)
    ref = [torch.zeros(shape, dtype=CACHE[mode]), torch.zeros(shape, dtype=CACHE[mode]),
           torch.zeros(NB, BS, KVH), torch.zeros(NB, BS, KVH)]
    store_kvcache_quant_per_token_head_ref(key, value, *ref, slots, BS, mode)
    got = _store_cuda(mode, key, value, torch.zeros(shape, dtype=CACHE[mode]),
                      torch.zeros(shape, dtype=CACHE[mode]), torch.zeros(NB, BS, KVH),
                      torch.zeros(NB, BS, KVH), slots, BS)
    q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
    cl = torch.tensor(lens, dtype=torch.int64)
    out = _decode_cuda(mode, q, *got, bt, cl, 0.09, H, KVH, D, BS)
    _close(out, paged_decode_ref(q, ref[0], ref[1], bt, cl, 0.09, H, KVH, D, BS, k_scales=ref[2],
                                 v_scales=ref[3]), torch.bfloat16)


def test_int8_step_in_cuda_graph():
    """INT8 append + decode captured once and replayed equal the eager result."""
    B, H, KVH, D, BS = 16, 32, 8, 128, 16
    g = torch.Generator().manual_seed(9)
    lens = torch.randint(1, 600, (B,), generator=g).tolist()
    q, kc, vc, ks, vs, bt, cl = _paged(B, H, KVH, D, BS, lens, "int8", seed=9, qdtype=torch.bfloat16)
    q, kc, vc, ks, vs, bt, cl = (t.cuda() for t in (q, kc, vc, ks, vs, bt, cl))
    nk = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16).cuda()
    nv = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16).cuda()
    slots = torch.tensor([int(bt[b, (n - 1) // BS]) * BS + (n - 1) % BS for b, n in enumerate(lens)],
                         dtype=torch.int64).cuda()

    def step():
        attn.store_kvcache_int8(nk, nv, kc, vc, ks, vs, slots, BS)
        return attn.paged_attention_decode_quantized(q, kc, vc, ks, vs, bt, cl, 0.088, H, KVH, D, BS,
                                                     "int8_per_token_head")

    eager = step().clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_out = step()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(static_out, eager)


PTH_CASES = ["outlier_q", "wide_scales", "peaked", "uniform_long"]


@pytest.mark.parametrize("mode", ["fp8", "int8"])
@pytest.mark.parametrize("case", PTH_CASES)
def test_decode_per_token_head_adversarial(mode, case):
    """Inputs that push the 8-bit decodes' arithmetic: queries with x100 outlier
    dimensions (the e4m3 hi + lo query split; int8's 1152 bias on S), per-(token, head)
    scales spread over 12 binades (the e4m3 kernel's per-warp power of two for V), a
    softmax concentrated on one token per sequence, and a uniform softmax over 16384
    tokens. Each must stay within the bf16 tolerance of the float64 oracle; the worst
    error / tolerance is printed."""
    H, KVH, D, BS = 32, 8, 128, 256
    seed = 101 + PTH_CASES.index(case) + (0 if mode == "fp8" else 50)
    lens = [16384, 16384] if case == "uniform_long" else [200, 1500, 2900, 777, 64, 2048]
    q, kc, vc, ks, vs, bt, cl = _paged(len(lens), H, KVH, D, BS, lens, mode, seed=seed,
                                       qdtype=torch.float32)
    g = torch.Generator().manual_seed(seed + 1)
    scale = 1.0 / math.sqrt(D)
    if case == "outlier_q":
        q[:, :, ::16] *= 100.0
    if case == "wide_scales":
        ks = torch.pow(2.0, torch.rand(ks.shape, generator=g) * 12 - 10)
        vs = torch.pow(2.0, torch.rand(vs.shape, generator=g) * 12 - 10)
    if case == "uniform_long":
        scale = 1e-6
    if case == "peaked":  # one token per sequence aligned with every query head of its kv head
        for b, n in enumerate(lens):
            t = int(torch.randint(0, n, (1,), generator=g))
            page, off = int(bt[b, t // BS]), t % BS
            for h in range(KVH):
                row = q[b, h * (H // KVH)] * 40
                kc[page, off, h] = (row.to(torch.float8_e4m3fn) if mode == "fp8"
                                    else row.round().clamp(-127, 127).to(torch.int8))
    q = q.to(torch.bfloat16)
    ref = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS, k_scales=ks, v_scales=vs)
    out = _decode_cuda(mode, q, kc, vc, ks, vs, bt, cl, scale, H, KVH, D, BS)
    atol, rtol = TOL[torch.bfloat16]
    margin = float(((out.double() - ref).abs() / (atol + rtol * ref.abs())).max())
    print(f"\nPTH_ADVERSARIAL {mode} {case}: max |err| {float((out.double() - ref).abs().max()):.3e}, "
          f"max |ref| {float(ref.abs().max()):.3e}, worst err/tol {margin:.4f}")
    assert margin <= 1.0
