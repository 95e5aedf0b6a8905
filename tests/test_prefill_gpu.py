"""Chunked-prefill / extend attention over the paged cache (paged_attention_prefill) on the
GPU against the CPU oracle paged_prefill_ref, which is pinned to the reference's
paged_attention_prefill_triton / _torch by tests/golden/prefill.npz.

Tolerances: bf16/fp16 queries atol 2e-2 / rtol 1e-2 (fp32 accumulation; P rounded to the
query dtype for the PV product), fp32 queries atol 2e-5 / rtol 1e-4."""
import math

import pytest
import torch

from conftest import golden, mkv_module
from oracle import paged_prefill_ref, varlen_prefill_ref

pytestmark = pytest.mark.gpu
attn = mkv_module("layers.attention")
TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (2e-2, 1e-2), torch.bfloat16: (2e-2, 1e-2)}


def make_case(ctx, chunk, H, KVH, D, BS, dtype, seed, cache="same", start=None):
    """Sequences whose last chunk[b] tokens of ctx[b] are the new queries (positions
    ctx - chunk .. ctx - 1), pages a random permutation."""
    g = torch.Generator().manual_seed(seed)
    B = len(ctx)
    need = [(n + BS - 1) // BS for n in ctx]
    NB = sum(need) + 3
    perm = torch.randperm(NB, generator=g)
    bt = torch.full((B, max(max(need), 1)), -1, dtype=torch.int32)
    pos = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[pos:pos + k].int()
        pos += k
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(chunk), 0).tolist()), dtype=torch.int32)
    positions = torch.cat([torch.arange(c - n, c) for c, n in zip(ctx, chunk)]).long()
    q = torch.randn(int(cu[-1]), H, D, generator=g).to(dtype)
    raw = torch.randn(2, NB, BS, KVH, D, generator=g)
    ks = vs = None
    if cache == "same":
        kc, vc = raw[0].to(dtype), raw[1].to(dtype)
    elif cache == "fp8_per_tensor":
        kc, vc = (raw[0] * 40).to(torch.float8_e4m3fn), (raw[1] * 40).to(torch.float8_e4m3fn)
        ks, vs = torch.tensor([0.021]), torch.tensor([0.032])
    else:
        if cache == "fp8_per_token_head":
            kc, vc = (raw[0] * 40).to(torch.float8_e4m3fn), (raw[1] * 40).to(torch.float8_e4m3fn)
        else:
            kc = (raw[0] * 40).round().clamp(-128, 127).to(torch.int8)
            vc = (raw[1] * 40).round().clamp(-128, 127).to(torch.int8)
        ks = torch.rand(NB, BS, KVH, generator=g) * 0.04 + 0.002
        vs = torch.rand(NB, BS, KVH, generator=g) * 0.04 + 0.002
    return q, kc, vc, bt, torch.tensor(ctx, dtype=torch.int64), cu, positions, ks, vs


def run(case, H, KVH, D, BS, scale, cache="same"):
    q, kc, vc, bt, cl, cu, pos, ks, vs = case
    mode = "auto" if cache == "same" else cache
    kw = {} if ks is None else dict(k_scale=ks.cuda(), v_scale=vs.cuda(), kv_cache_dtype=mode)
    out = attn.paged_attention_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), cu.cuda(),
                                       pos.cuda(), scale, H, KVH, D, BS, **kw)
    torch.cuda.synchronize()
    if ks is None:
        ref = paged_prefill_ref(q, kc, vc, bt, cl, cu, pos, scale, H, KVH, BS)
    elif cache == "fp8_per_tensor":
        ref = paged_prefill_ref(q, kc, vc, bt, cl, cu, pos, scale, H, KVH, BS, k_scale=ks, v_scale=vs)
    else:
        ref = paged_prefill_ref(q, kc, vc, bt, cl, cu, pos, scale, H, KVH, BS, k_scales=ks, v_scales=vs)
    return out.cpu(), ref


def close(out, ref, dtype):
    atol, rtol = TOL[dtype]
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(out), nan), "NaN pattern differs"
    diff = (out.double() - ref)[~nan].abs()
    assert bool((diff <= atol + rtol * ref[~nan].abs()).all()), f"max abs err {float(diff.max()):.3e}"


@pytest.fixture(params=["auto", "1", "2"])
def qtiles(request, monkeypatch):
    """The tensor-core prefill's query tiles per CTA: the library's choice, or forced to
    one or two (MKV_PREFILL_QTILES, read per call)."""
    if request.param == "auto":
        monkeypatch.delenv("MKV_PREFILL_QTILES", raising=False)
    else:
        monkeypatch.setenv("MKV_PREFILL_QTILES", request.param)
    return request.param


CTX = [300, 64, 1, 130, 17, 700]
CHUNK = [300, 5, 1, 65, 17, 256]  # full prefill, short extend, single token, chunked


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("H,KVH", [(8, 8), (16, 4), (32, 2), (6, 2)])
@pytest.mark.parametrize("BS", [16, 256])
def test_prefill_matches_oracle(dtype, H, KVH, BS, qtiles):
    D = 128
    case = make_case(CTX, CHUNK, H, KVH, D, BS, dtype, seed=H * 3 + KVH + BS)
    out, ref = run(case, H, KVH, D, BS, 1.0 / math.sqrt(D))
    close(out, ref, dtype)


@pytest.mark.parametrize("D", [64, 96, 256])
def test_prefill_other_head_dims(D):
    case = make_case(CTX, CHUNK, 8, 2, D, 16, torch.bfloat16, seed=D)
    out, ref = run(case, 8, 2, D, 16, 1.0 / math.sqrt(D))
    close(out, ref, torch.bfloat16)


QUANT = ["fp8_per_tensor", "fp8_per_token_head", "int8_per_token_head"]


@pytest.fixture(params=["scratch", "in-kernel"])
def page_conversion(request, monkeypatch):
    """8-bit caches with long chunks: pages converted once into the workspace (the
    default), or tile by tile inside the attention kernel (MKV_PREFILL_WORKSPACE=0)."""
    monkeypatch.setenv("MKV_PREFILL_WORKSPACE", "1" if request.param == "scratch" else "0")
    return request.param


@pytest.mark.parametrize("cache", QUANT)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("BS", [16, 256])
def test_prefill_quantised_caches(cache, dtype, BS):
    """Quantised caches dequantised in the kernel (the reference's TODO): 16-bit queries
    take the tcgen05 kernel (8-bit tiles converted in shared memory), fp32 queries the
    CUDA-core kernel."""
    case = make_case(CTX, CHUNK, 16, 4, 128, BS, dtype, seed=7 + BS, cache=cache)
    out, ref = run(case, 16, 4, 128, BS, 0.0883, cache=cache)
    close(out, ref, dtype)


@pytest.mark.parametrize("cache", QUANT)
@pytest.mark.parametrize("BS", [16, 64, 256])
def test_prefill_quantised_missing_pages(cache, BS, page_conversion):
    """Missing and out-of-range pages with 8-bit caches: their rows convert to zeros."""
    case = list(make_case([700, 600], [300, 600], 16, 4, 128, BS, torch.bfloat16, seed=BS + 1, cache=cache))
    bt = case[3].clone()
    bt[0, 1] = -1
    bt[1, 0] = 10 ** 6
    case[3] = bt
    out, ref = run(tuple(case), 16, 4, 128, BS, 0.09, cache=cache)
    assert torch.isnan(ref).any()
    close(out, ref, torch.bfloat16)


@pytest.mark.parametrize("cache", QUANT)
def test_prefill_quantised_long_chunk(cache, page_conversion):
    """A 2048-token chunk after a 4096-token prefix over an 8-bit cache, GQA 4."""
    case = make_case([6144, 900], [2048, 900], 32, 8, 128, 256, torch.bfloat16, seed=13, cache=cache)
    out, ref = run(case, 32, 8, 128, 256, 1.0 / math.sqrt(128), cache=cache)
    close(out, ref, torch.bfloat16)


def test_prefill_invalid_pages_and_empty_rows(qtiles):
    """-1 pages inside a context are skipped; a query whose visible range holds only
    missing pages gives NaN."""
    case = list(make_case([40, 20], [40, 10], 8, 2, 128, 16, torch.bfloat16, seed=3))
    bt = case[3].clone()
    bt[0, 1] = -1            # tokens 16..31 of sequence 0 missing
    bt[1, 0] = 10 ** 6       # tokens 0..15 of sequence 1 out of range: its rows at
                             # positions 10..15 see nothing
    case[3] = bt
    out, ref = run(tuple(case), 8, 2, 128, 16, 0.09)
    assert torch.isnan(ref).any()  # sequence 1's early rows see only missing pages
    close(out, ref, torch.bfloat16)


@pytest.mark.parametrize("BS", [16, 64, 256])
def test_prefill_missing_pages_by_block_size(BS, qtiles):
    """Missing pages that cover a part of a 128-token tile (BS 16, 64) or a whole tile and
    more (BS 256), on top of the causal edge."""
    case = list(make_case([700, 600], [300, 600], 16, 4, 128, BS, torch.bfloat16, seed=BS))
    bt = case[3].clone()
    bt[0, 1] = -1        # sequence 0: tokens BS .. 2 BS - 1 missing
    bt[1, 0] = 10 ** 6   # sequence 1: its first page out of range
    case[3] = bt
    out, ref = run(tuple(case), 16, 4, 128, BS, 0.09)
    assert torch.isnan(ref).any()
    close(out, ref, torch.bfloat16)


def test_prefill_long_chunk(qtiles):
    """A 2048-token chunk extending a 4096-token prefix (many KV tiles, causal edge in
    the middle of a tile), GQA 4."""
    case = make_case([6144, 900], [2048, 900], 32, 8, 128, 256, torch.bfloat16, seed=11)
    out, ref = run(case, 32, 8, 128, 256, 1.0 / math.sqrt(128))
    close(out, ref, torch.bfloat16)


def test_golden_prefill_through_cuda():
    g = golden("prefill")
    t = lambda k: torch.from_numpy(g[k])
    H, KVH, BS = int(g["num_heads"]), int(g["num_kv_heads"]), int(g["block_size"])
    q = t("query")
    out = attn.paged_attention_prefill(q.cuda(), t("k_cache").cuda(), t("v_cache").cuda(),
                                       t("block_tables").cuda(), t("context_lens").cuda(),
                                       t("cu_seqlens_q").cuda(), t("positions").cuda(), float(g["scale"]),
                                       H, KVH, q.shape[2], BS).cpu()
    close(out, t("out").double(), torch.float32)


def test_prefill_matches_decode_for_last_token(qtiles):
    """For each sequence, the prefill row of its last context token equals the decode of
    that sequence over the same cache."""
    H, KVH, D, BS = 32, 8, 128, 16
    case = make_case(CTX, CHUNK, H, KVH, D, BS, torch.bfloat16, seed=5)
    q, kc, vc, bt, cl, cu, pos, _, _ = case
    out = attn.paged_attention_prefill(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), cu.cuda(),
                                       pos.cuda(), 0.09, H, KVH, D, BS)
    last = (cu[1:] - 1).long()
    dec = attn.paged_attention_decode(q[last].cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), 0.09,
                                      H, KVH, D, BS)
    torch.cuda.synchronize()
    close(out[last.cuda()].cpu(), dec.cpu().double(), torch.bfloat16)


# ------------------------------------------------------------ contiguous (full) prefill
def test_varlen_prefill_golden_fp32():
    """flash_attention_prefill on the reference's fixture (fp32, CUDA-core path)."""
    g = golden("varlen_prefill")
    out = attn.flash_attention_prefill(
        torch.from_numpy(g["query"]).cuda(), torch.from_numpy(g["key"]).cuda(),
        torch.from_numpy(g["value"]).cuda(), torch.from_numpy(g["cu_seqlens"]).cuda(),
        float(g["scale"]), int(g["num_heads"]), int(g["num_kv_heads"]), g["query"].shape[2])
    assert torch.allclose(out.cpu().double(), torch.from_numpy(g["out"]).double(), atol=2e-5, rtol=1e-4)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,KVH,D", [(32, 8, 128), (16, 8, 128), (8, 2, 64)])
@pytest.mark.parametrize("give_max", [False, True])
def test_varlen_prefill_against_oracle(dtype, H, KVH, D, give_max):
    """Ragged whole prompts (1 token, page-boundary lengths, 700) against varlen_prefill_ref,
    with the longest length read from cu_seqlens or given as an upper bound."""
    g = torch.Generator().manual_seed(H + D)
    lens = [1, 128, 129, 700, 37, 256, 5]
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0)), dtype=torch.int32)
    T = int(cu[-1])
    q = torch.randn(T, H, D, generator=g).to(dtype)
    k = torch.randn(T, KVH, D, generator=g).to(dtype)
    v = torch.randn(T, KVH, D, generator=g).to(dtype)
    scale = 1.0 / math.sqrt(D)
    out = attn.flash_attention_prefill(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), scale, H, KVH, D,
                                       max_seqlen=1024 if give_max else None)
    ref = varlen_prefill_ref(q, k, v, cu, scale, H, KVH)
    assert torch.allclose(out.cpu().double(), ref, atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("mode", ["auto", "fp8_per_tensor", "int8_per_token_head"])
def test_attention_full_prefill_uses_contiguous_kv(mode):
    """Attention.forward on a batch of whole prompts (context.is_full_prefill, no block
    tables, as prepare_prefill sets it without a prefix-cache hit): the output is the
    causal attention over the step's own q/k/v (attention.py:1771), with the K/V appended
    to the cache; and with no cache at all (the runner's warm-up) it is the same."""
    kvc = mkv_module("engine.kv_cache")
    ctx = mkv_module("utils.context")
    H, KVH, D, BS = 16, 8, 128, 16
    lens = [3, 40, 17]
    cu = torch.tensor([0, 3, 43, 60], dtype=torch.int32)
    T = 60
    g = torch.Generator().manual_seed(3)
    q = torch.randn(T, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(T, KVH, D, generator=g).to(torch.bfloat16)
    v = torch.randn(T, KVH, D, generator=g).to(torch.bfloat16)
    ref = varlen_prefill_ref(q, k, v, cu, 1.0 / math.sqrt(D), H, KVH)
    layer = attn.Attention(H, D, scale=1.0, num_kv_heads=KVH, block_size=BS)
    slots = torch.arange(T, dtype=torch.int64)
    for with_cache in (False, True):
        if with_cache:
            cache = kvc.allocate_kv_cache(1, 8, BS, KVH, D, mode)
            kvc.bind_kv_cache(layer.modules(), cache)
        ctx.set_context(True, cu_seqlens_q=cu.cuda(), cu_seqlens_k=cu.cuda(), max_seqlen_q=40,
                        max_seqlen_k=40, slot_mapping=slots.cuda() if with_cache else None,
                        is_full_prefill=True)
        o = layer(q.cuda(), k.cuda(), v.cuda())
        torch.cuda.synchronize()
        ctx.reset_context()
        assert o.shape == (T, H * D)
        assert torch.allclose(o.view(T, H, D).cpu().double(), ref, atol=2e-2, rtol=1e-2)
        if with_cache and mode == "auto":  # the step's K/V were appended too
            assert torch.equal(cache.kv[0, 0].reshape(-1, KVH, D)[:T].cpu(), k)
