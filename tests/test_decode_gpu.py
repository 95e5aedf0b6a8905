"""Paged-attention decode on the GPU through the C ABI against the CPU oracle
(token-level restatement of the reference kernel, float64), the BASELINE
configurations 3 and 4 at full size included (every sequence).

Tolerances: bf16/fp16 outputs atol 2e-2 / rtol 1e-2 (the BASELINE bar, fp32
accumulation); fp32 outputs atol 2e-5 / rtol 1e-4."""
import math

import numpy as np
import pytest
import torch

from conftest import golden, mkv_module
from oracle import paged_decode_ref

pytestmark = pytest.mark.gpu
attn = mkv_module("layers.attention")
wl = mkv_module("workloads")

TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (2e-2, 1e-2), torch.bfloat16: (2e-2, 1e-2)}


def make_paged(B, H, KVH, D, BS, lens, dtype, seed, maxb=None, fp8=False, spare=5):
    g = torch.Generator().manual_seed(seed)
    need = [(n + BS - 1) // BS for n in lens]
    maxb = maxb if maxb is not None else max(max(need), 1)
    NB = sum(need) + spare
    perm = torch.randperm(NB, generator=g)
    bt = torch.full((B, maxb), -1, dtype=torch.int32)
    pos = 0
    for b, k in enumerate(need):
        kk = min(k, maxb)
        bt[b, :kk] = perm[pos:pos + kk].int()
        pos += k
    q = torch.randn(B, H, D, generator=g).to(dtype)
    if fp8:
        kc = (torch.randn(NB, BS, KVH, D, generator=g) * 30).to(torch.float8_e4m3fn)
        vc = (torch.randn(NB, BS, KVH, D, generator=g) * 30).to(torch.float8_e4m3fn)
    else:
        kc = torch.randn(NB, BS, KVH, D, generator=g).to(dtype)
        vc = torch.randn(NB, BS, KVH, D, generator=g).to(dtype)
    return q, kc, vc, bt, torch.tensor(lens, dtype=torch.int64)


def run_cuda(q, kc, vc, bt, cl, scale, H, KVH, D, BS, ks=None, vs=None, splits=0):
    if ks is None:
        return attn.paged_attention_decode(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), cl.cuda(), scale,
                                           H, KVH, D, BS, num_splits=splits).cpu()
    return attn.paged_attention_decode_quantized(q.cuda(), kc.cuda(), vc.cuda(), ks.cuda(), vs.cuda(),
                                                 bt.cuda(), cl.cuda(), scale, H, KVH, D, BS,
                                                 "fp8_per_tensor", num_splits=splits).cpu()


def assert_close(out, ref, dtype):
    atol, rtol = TOL[dtype]
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(out), nan), "NaN pattern differs"
    diff = (out.double() - ref)[~nan].abs()
    bound = atol + rtol * ref[~nan].abs()
    assert bool((diff <= bound).all()), f"max abs err {float(diff.max()):.3e}"


LENS = [1, 16, 17, 63, 64, 65, 200, 511, 0, 300]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("H,KVH", [(8, 8), (16, 8), (32, 8), (8, 1), (32, 2), (64, 2)])
@pytest.mark.parametrize("BS", [16, 256])
def test_decode_matches_oracle(dtype, H, KVH, BS):
    D = 128
    q, kc, vc, bt, cl = make_paged(len(LENS), H, KVH, D, BS, LENS, dtype, seed=H * 7 + KVH + BS)
    scale = 1.0 / math.sqrt(D)
    ref = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS)
    assert_close(run_cuda(q, kc, vc, bt, cl, scale, H, KVH, D, BS), ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [64, 256, 96])
def test_decode_other_head_dims(dtype, D):
    H, KVH, BS = 8, 2, 16
    q, kc, vc, bt, cl = make_paged(len(LENS), H, KVH, D, BS, LENS, dtype, seed=D)
    scale = 1.0 / math.sqrt(D)
    ref = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS)
    assert_close(run_cuda(q, kc, vc, bt, cl, scale, H, KVH, D, BS), ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("H,KVH", [(32, 8), (16, 8), (32, 2)])
def test_decode_fp8_matches_oracle(dtype, H, KVH):
    D, BS = 128, 16
    q, kc, vc, bt, cl = make_paged(len(LENS), H, KVH, D, BS, LENS, dtype, seed=3 + H, fp8=True)
    ks = torch.tensor([0.0213623046875])
    vs = torch.tensor([0.031982421875])
    scale = 1.0 / math.sqrt(D)
    ref = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS, k_scale=ks, v_scale=vs)
    assert_close(run_cuda(q, kc, vc, bt, cl, scale, H, KVH, D, BS, ks, vs), ref, dtype)


def test_decode_bf16_query_with_large_values_fp8():
    """bf16 queries far outside f16 range still work on the FP8 path (power-of-two
    rescaling of the query fragments)."""
    D, BS, H, KVH = 128, 16, 8, 2
    q, kc, vc, bt, cl = make_paged(4, H, KVH, D, BS, [40, 90, 7, 128], torch.bfloat16, seed=9, fp8=True)
    q = (q.float() * 1e6).to(torch.bfloat16)
    ks, vs = torch.tensor([0.01]), torch.tensor([0.02])
    scale = 1e-7
    ref = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS, k_scale=ks, v_scale=vs)
    assert_close(run_cuda(q, kc, vc, bt, cl, scale, H, KVH, D, BS, ks, vs), ref, torch.bfloat16)


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 64])
@pytest.mark.parametrize("fp8", [False, True])
def test_decode_forced_splits(splits, fp8):
    D, BS, H, KVH = 128, 16, 32, 8
    lens = [1000, 1, 64, 777, 0, 129]
    q, kc, vc, bt, cl = make_paged(len(lens), H, KVH, D, BS, lens, torch.bfloat16, seed=splits, fp8=fp8)
    ks = torch.tensor([0.02]) if fp8 else None
    vs = torch.tensor([0.03]) if fp8 else None
    ref = paged_decode_ref(q, kc, vc, bt, cl, 0.0883, H, KVH, D, BS, k_scale=ks, v_scale=vs)
    assert_close(run_cuda(q, kc, vc, bt, cl, 0.0883, H, KVH, D, BS, ks, vs, splits=splits), ref,
                 torch.bfloat16)


def test_decode_invalid_pages_inside_context():
    """-1 (and out-of-range) page entries inside a context skip those tokens, like the
    reference kernel; a context whose pages are all invalid yields NaN."""
    D, BS, H, KVH = 128, 16, 8, 2
    lens = [100, 50, 30]
    q, kc, vc, bt, cl = make_paged(3, H, KVH, D, BS, lens, torch.bfloat16, seed=4)
    bt[0, 2] = -1
    bt[1, 1] = 10 ** 6       # out of range: treated as no page
    bt[2, :2] = -1           # every page of sequence 2 invalid
    ref = paged_decode_ref(q, kc, vc, bt, cl, 0.1, H, KVH, D, BS)
    out = run_cuda(q, kc, vc, bt, cl, 0.1, H, KVH, D, BS)
    assert torch.isnan(out[2]).all()
    assert_close(out, ref, torch.bfloat16)


def test_decode_noncontiguous_query_and_int32_lengths():
    D, BS, H, KVH = 128, 16, 16, 4
    q, kc, vc, bt, cl = make_paged(5, H, KVH, D, BS, [5, 60, 33, 100, 17], torch.bfloat16, seed=8)
    qbig = torch.randn(5, 3 * H, D).to(torch.bfloat16)
    qbig[:, H:2 * H] = q
    qv = qbig.cuda()[:, H:2 * H]
    assert not qv.is_contiguous()
    out = attn.paged_attention_decode(qv, kc.cuda(), vc.cuda(), bt.cuda(), cl.int().cuda(), 0.09,
                                      H, KVH, D, BS).cpu()
    assert_close(out, paged_decode_ref(q, kc, vc, bt, cl, 0.09, H, KVH, D, BS), torch.bfloat16)


def test_golden_decode_small_through_cuda():
    g = golden("decode_small")
    H, KVH, BS = int(g["num_heads"]), int(g["num_kv_heads"]), int(g["block_size"])
    q = torch.from_numpy(g["query"])
    out = run_cuda(q, torch.from_numpy(g["k_cache"]), torch.from_numpy(g["v_cache"]),
                   torch.from_numpy(g["block_tables"]), torch.from_numpy(g["context_lens"]),
                   float(g["scale"]), H, KVH, q.shape[2], BS)
    assert_close(out, torch.from_numpy(g["out"]).double(), torch.float32)


def test_golden_decode_fp8_through_cuda():
    g = golden("decode_fp8")
    H, KVH, BS = int(g["num_heads"]), int(g["num_kv_heads"]), int(g["block_size"])
    q = torch.from_numpy(g["query"])
    out = run_cuda(q, torch.from_numpy(g["k_cache_e4m3"]).view(torch.float8_e4m3fn),
                   torch.from_numpy(g["v_cache_e4m3"]).view(torch.float8_e4m3fn),
                   torch.from_numpy(g["block_tables"]), torch.from_numpy(g["context_lens"]),
                   float(g["scale"]), H, KVH, q.shape[2], BS, torch.from_numpy(g["k_scale"]),
                   torch.from_numpy(g["v_scale"]))
    assert_close(out, torch.from_numpy(g["out"]).double(), torch.float32)


def test_golden_config1_through_cuda():
    from golden.make_golden import config1_inputs
    g = golden("decode_config1")
    inp = config1_inputs(int(g["seed"]))
    out = run_cuda(torch.from_numpy(inp["query"]), torch.from_numpy(inp["k_cache"]),
                   torch.from_numpy(inp["v_cache"]), torch.from_numpy(inp["block_tables"]),
                   torch.from_numpy(inp["context_lens"]), float(g["scale"]), inp["num_heads"],
                   inp["num_kv_heads"], inp["head_dim"], inp["block_size"])
    assert_close(out, torch.from_numpy(g["out"]).double(), torch.float32)


# ------------------------------------------------------------------ full-size configs
def torch_reference(w, seqs):
    """float32 attention on the GPU for the given sequences (dequantised for FP8)."""
    H, KVH, D, BS = w.num_heads, w.num_kv_heads, w.head_dim, w.block_size
    G = H // KVH
    out = []
    for b in seqs:
        n = int(w.context_lens[b])
        pages = w.block_tables[b, :(n + BS - 1) // BS].long()
        K = w.k_cache[pages].reshape(-1, KVH, D)[:n].float()
        V = w.v_cache[pages].reshape(-1, KVH, D)[:n].float()
        if w.fp8:
            K, V = K * w.k_scale, V * w.v_scale
        qb = w.query[b].float().view(KVH, G, D)
        s = torch.einsum("hgd,thd->hgt", qb, K) * w.scale
        out.append(torch.einsum("hgt,thd->hgd", torch.softmax(s, -1), V).reshape(H, D))
    return torch.stack(out)


def _decode_w(w, splits=0):
    if w.fp8:
        return attn.paged_attention_decode_quantized(
            w.query, w.k_cache, w.v_cache, w.k_scale, w.v_scale, w.block_tables, w.context_lens,
            w.scale, w.num_heads, w.num_kv_heads, w.head_dim, w.block_size, "fp8_per_tensor",
            num_splits=splits)
    return attn.paged_attention_decode(w.query, w.k_cache, w.v_cache, w.block_tables,
                                       w.context_lens, w.scale, w.num_heads, w.num_kv_heads,
                                       w.head_dim, w.block_size, num_splits=splits)


def oracle_over_batch(w, chunk):
    """The float64 oracle (paged_decode_ref) over every sequence of a workload, `chunk`
    sequences at a time: each chunk's pages are gathered into a compact CPU cache and
    its block tables renumbered, so host memory stays bounded at full size."""
    B, BS = w.query.shape[0], w.block_size
    out = torch.empty(B, w.num_heads, w.head_dim, dtype=torch.float64)
    for s in range(0, B, chunk):
        e = min(B, s + chunk)
        bt = w.block_tables[s:e]
        pages = torch.unique(bt[bt >= 0])
        remap = torch.full((w.k_cache.shape[0],), -1, dtype=torch.int32, device=bt.device)
        remap[pages.long()] = torch.arange(pages.numel(), dtype=torch.int32, device=bt.device)
        bt_c = torch.where(bt >= 0, remap[bt.clamp(min=0).long()], bt).cpu()
        kc, vc = w.k_cache[pages.long()].cpu(), w.v_cache[pages.long()].cpu()
        ks = w.k_scale.cpu() if w.fp8 else None
        vs = w.v_scale.cpu() if w.fp8 else None
        out[s:e] = paged_decode_ref(w.query[s:e].cpu(), kc, vc, bt_c, w.context_lens[s:e].cpu(),
                                    w.scale, w.num_heads, w.num_kv_heads, w.head_dim, BS,
                                    k_scale=ks, v_scale=vs)
    return out


def tolerance_margin(got, ref, atol, rtol):
    """max over elements of |got - ref| / (atol + rtol |ref|): <= 1 passes allclose."""
    return float(((got.double() - ref).abs() / (atol + rtol * ref.abs())).max())


@pytest.mark.parametrize("cfg", ["config3", "config4"])
def test_full_size_config(cfg):
    """Configs 3 (bf16, 256 sequences) and 4 (FP8, 64 x 32768 tokens) at full size:
    every sequence against the float64 oracle, and the whole batch for split-count
    invariance. Prints the worst error as a fraction of the tolerance."""
    w = getattr(wl, cfg)(seed=1, with_append=False)
    out = _decode_w(w)
    torch.cuda.synchronize()
    assert not torch.isnan(out).any()
    ref = oracle_over_batch(w, 16 if cfg == "config3" else 2)
    atol, rtol = TOL[torch.bfloat16]
    got = out.cpu()
    margin = tolerance_margin(got, ref, atol, rtol)
    err = float((got.double() - ref).abs().max())
    print(f"\nFULL_SIZE_PARITY {cfg}: {w.query.shape[0]} sequences, max |err| {err:.3e}, "
          f"worst err/tol {margin:.4f} (atol {atol}, rtol {rtol})")
    assert margin <= 1.0
    # split-count invariance over the whole batch: one split vs the automatic plan
    one = _decode_w(w, splits=1)
    assert torch.allclose(one.float(), out.float(), atol=atol, rtol=rtol)


def test_decode_step_in_cuda_graph():
    """Append + decode (bf16 and FP8) captured once and replayed equal the eager result."""
    for fp8 in (False, True):
        w = wl.decode_workload("g", 16, 32, 8, 128, 16, [int(x) for x in torch.randint(1, 600, (16,))],
                               fp8=fp8, seed=5)
        ks = torch.ones(1, device="cuda") if fp8 else None
        vs = torch.ones(1, device="cuda") if fp8 else None

        def step():
            if fp8:
                attn.store_kvcache_fp8(w.new_k, w.new_v, w.k_cache, w.v_cache, ks, vs, w.slot_mapping,
                                       w.block_size, "fp8_per_tensor")
                return attn.paged_attention_decode_quantized(
                    w.query, w.k_cache, w.v_cache, ks, vs, w.block_tables, w.context_lens, w.scale,
                    w.num_heads, w.num_kv_heads, w.head_dim, w.block_size, "fp8_per_tensor")
            attn.store_kvcache(w.new_k, w.new_v, w.k_cache, w.v_cache, w.slot_mapping, w.block_size)
            return _decode_w(w)

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


# ------------------------------------------------------------------ balanced schedule
def _balanced_case(case, fp8):
    g = torch.Generator().manual_seed(11)
    if case == "one_long":        # one unit per kv head, each shared by ~80 CTAs
        return wl.decode_workload(case, 1, 32, 8, 128, 16, [20000], fp8=fp8, seed=21, with_append=False)
    if case == "many_ragged":     # 600 sequences, 10% empty, segments beyond the staged table
        lens = torch.randint(0, 3000, (600,), generator=g)
        lens[torch.rand(600, generator=g) < 0.1] = 0
        return wl.decode_workload(case, 600, 32, 8, 128, 16, lens.tolist(), fp8=fp8, seed=22,
                                  with_append=False)
    if case == "wide_group":      # 32 query heads per kv head: two head groups per unit
        return wl.decode_workload(case, 7, 64, 2, 128, 256, [9000, 1, 0, 4097, 128, 65, 30000],
                                  fp8=fp8, seed=23, with_append=False)
    if case == "unit_major":      # 32 kv heads do not divide a 444-CTA grid: unit-major order
        lens = torch.randint(0, 2500, (40,), generator=g).tolist()
        return wl.decode_workload(case, 40, 32, 32, 128, 16, lens, fp8=fp8, seed=25, with_append=False)
    # a table wide enough that the merge bound (128 partials per unit) sets the CTA share
    return wl.decode_workload(case, 2, 8, 1, 128, 256, [100000, 3], fp8=fp8, seed=24, with_append=False)


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("case", ["one_long", "many_ragged", "wide_group", "unit_major", "very_long"])
def test_balanced_schedule(case, fp8):
    """The automatic (balanced, persistent) schedule against a float32 torch reference on
    every sequence, and against the one-split plan over the whole batch."""
    w = _balanced_case(case, fp8)
    out = _decode_w(w)
    torch.cuda.synchronize()
    atol, rtol = TOL[torch.bfloat16]
    lens = w.context_lens.tolist()
    live = [b for b, n in enumerate(lens) if n > 0]
    empty = [b for b, n in enumerate(lens) if n == 0]
    assert torch.isnan(out[empty]).all() if empty else True
    assert not torch.isnan(out[live]).any()
    for i in range(0, len(live), 64):
        seqs = live[i:i + 64]
        assert torch.allclose(out[seqs].float(), torch_reference(w, seqs), atol=atol, rtol=rtol)
    one = _decode_w(w, splits=1)
    assert torch.allclose(one[live].float(), out[live].float(), atol=atol, rtol=rtol)
    again = _decode_w(w)  # counters were left at zero: a second launch agrees bit for bit
    assert torch.equal(torch.nan_to_num(again, nan=7.0), torch.nan_to_num(out, nan=7.0))


def test_balanced_schedule_counts_invalid_pages_once():
    """Out-of-range page entries are counted once per (sequence, entry) whatever the
    schedule, here on segments longer than the staged block-table slice."""
    lib = mkv_module("_lib").load()
    w = wl.decode_workload("inv", 3, 8, 2, 128, 16, [4000, 2500, 700], seed=31, with_append=False)
    w.block_tables[0, 5] = 10 ** 6
    w.block_tables[0, 200] = -7
    w.block_tables[1, 3] = 10 ** 6
    for splits in (0, 1, 5):
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        out = torch.empty_like(w.query)
        n = lib.mkv_paged_decode_workspace_bytes(3, 8, 2, 128, 16, w.block_tables.shape[1], splits)
        ws = torch.empty(max(n, 1), dtype=torch.uint8, device="cuda")
        st = lib.mkv_paged_decode(
            w.query.data_ptr(), w.query.stride(0), w.query.stride(1), 2, w.k_cache.data_ptr(),
            w.v_cache.data_ptr(), 2, w.k_cache.shape[0], 16, w.block_tables.data_ptr(), 0,
            w.block_tables.stride(0), w.block_tables.shape[1], w.context_lens.data_ptr(), 1, 3, 8, 2,
            128, w.scale, out.data_ptr(), out.stride(0), out.stride(1), ws.data_ptr(), n, splits,
            cnt.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert st == 0, lib.mkv_last_error()
        torch.cuda.synchronize()
        assert int(cnt) == 3, (splits, int(cnt))


# ------------------------------------------------------------------ launch options
@pytest.mark.parametrize("fp8", [False, True])
def test_overlapped_step_equals_serial_step(fp8):
    """The decode launched to overlap the append before it (programmatic dependent
    launch) reads what the append wrote: eager and CUDA-graph replays equal the serial
    step bit for bit, the FP8 scale calibrated by the append's first call included."""
    lens = [int(x) for x in torch.randint(1, 3000, (24,), generator=torch.Generator().manual_seed(9))]
    outs = []
    for overlap in (False, True, True):
        w = wl.decode_workload("ovl", 24, 32, 8, 128, 16, lens, fp8=fp8, seed=41)
        ks = torch.ones(1, device="cuda") if fp8 else None  # sentinel: the first append calibrates
        vs = torch.ones(1, device="cuda") if fp8 else None

        def step():
            if fp8:
                attn.store_kvcache_fp8(w.new_k, w.new_v, w.k_cache, w.v_cache, ks, vs, w.slot_mapping,
                                       w.block_size, "fp8_per_tensor")
                return attn.paged_attention_decode_quantized(
                    w.query, w.k_cache, w.v_cache, ks, vs, w.block_tables, w.context_lens, w.scale,
                    w.num_heads, w.num_kv_heads, w.head_dim, w.block_size, "fp8_per_tensor",
                    overlap_previous=overlap)
            attn.store_kvcache(w.new_k, w.new_v, w.k_cache, w.v_cache, w.slot_mapping, w.block_size)
            return attn.paged_attention_decode(w.query, w.k_cache, w.v_cache, w.block_tables,
                                               w.context_lens, w.scale, w.num_heads, w.num_kv_heads,
                                               w.head_dim, w.block_size, overlap_previous=overlap)

        if len(outs) < 2:
            outs.append(step().clone())
        else:  # captured: the graph's first replay does the calibration
            graph = torch.cuda.CUDAGraph()
            with fp8_suspended():
                step()  # warm-up without calibrating (allocates the scratch)
            torch.cuda.synchronize()
            with torch.cuda.graph(graph):
                static_out = step()
            graph.replay()
            graph.replay()
            torch.cuda.synchronize()
            outs.append(static_out.clone())
        torch.cuda.synchronize()
    assert torch.equal(torch.nan_to_num(outs[0], nan=3.0), torch.nan_to_num(outs[1], nan=3.0))
    assert torch.equal(torch.nan_to_num(outs[0], nan=3.0), torch.nan_to_num(outs[2], nan=3.0))


def fp8_suspended():
    return attn.fp8_calibration_suspended()


def test_shared_counter_buffer_across_shapes():
    """Decodes of different shapes and split counts, back to back on one stream, sharing
    the wrapper's counter buffer (zeroed once, never cleared again) and workspace: each
    equals the same decode with the library clearing fresh counters."""
    lib = mkv_module("_lib").load()
    cases = [(5, 32, 8, 16, [700, 3, 4000, 1, 128], 0), (3, 8, 2, 256, [9000, 17, 600], 4),
             (40, 16, 16, 16, [int(x) for x in torch.randint(0, 900, (40,))], 0),
             (2, 64, 2, 256, [30000, 5], 0), (7, 32, 8, 16, [333] * 7, 2)]
    for i, (B, H, KVH, BS, lens, splits) in enumerate(cases * 2):
        w = wl.decode_workload("ctr", B, H, KVH, 128, BS, lens, seed=60 + i, with_append=False)
        got = attn.paged_attention_decode(w.query, w.k_cache, w.v_cache, w.block_tables,
                                          w.context_lens, w.scale, H, KVH, 128, BS, num_splits=splits)
        out = torch.empty_like(w.query)
        n = lib.mkv_paged_decode_workspace_bytes(B, H, KVH, 128, BS, w.block_tables.shape[1], splits)
        ws = torch.full((max(n, 1),), 0xAB, dtype=torch.uint8, device="cuda")  # dirty
        st = lib.mkv_paged_decode(
            w.query.data_ptr(), w.query.stride(0), w.query.stride(1), 2, w.k_cache.data_ptr(),
            w.v_cache.data_ptr(), 2, w.k_cache.shape[0], BS, w.block_tables.data_ptr(), 0,
            w.block_tables.stride(0), w.block_tables.shape[1], w.context_lens.data_ptr(), 1, B, H,
            KVH, 128, w.scale, out.data_ptr(), out.stride(0), out.stride(1), ws.data_ptr(), n, splits,
            None, torch.cuda.current_stream().cuda_stream)
        assert st == 0, lib.mkv_last_error()
        torch.cuda.synchronize()
        assert torch.equal(torch.nan_to_num(got, nan=5.0), torch.nan_to_num(out, nan=5.0)), i


def test_decode_ex_rejects_bad_arguments():
    lib = mkv_module("_lib").load()
    t = torch.zeros(64, dtype=torch.float32, device="cuda")
    p = t.data_ptr()
    base = [p, 4096, 128, 2, p, p]
    tail = [1, 16, p, 0, 1, 1, p, 1, 1, 8, 2, 128, 0.1, p, 4096, 128, None, 0, None, 0, 0]
    stream = torch.cuda.current_stream().cuda_stream
    # unknown flag bits
    st = lib.mkv_paged_decode_ex(*base, 2, None, None, None, None, *tail, 9, None, stream)
    assert st == mkv_module("_lib").ERR_INVALID_ARGUMENT and b"flags" in lib.mkv_last_error()
    # per-tensor and per-(token, head) scales together
    st = lib.mkv_paged_decode_ex(*base, 3, p, p, p, p, *tail, 0, None, stream)
    assert st == mkv_module("_lib").ERR_INVALID_ARGUMENT
    # scales for an unquantised cache
    st = lib.mkv_paged_decode_ex(*base, 2, p, p, None, None, *tail, 0, None, stream)
    assert st == mkv_module("_lib").ERR_INVALID_ARGUMENT


# ------------------------------------------------------------------ FP8 operand split
def _fp8_cache(n_tokens, kvh, d, g, fill):
    x = fill(torch.randn(n_tokens, kvh, d, generator=g))
    return x.clamp(-448, 448).to(torch.float8_e4m3fn)


@pytest.mark.parametrize("case", ["peaked", "uniform_32k", "wide_v", "outlier_q", "tiny_scores"])
def test_decode_fp8_adversarial_ranges(case):
    """The FP8-MMA kernel splits the query and P into e4m3 hi + lo parts (about 8
    significant bits each, like bf16) where the reference dequantises to fp32 and dots in
    fp32. These inputs push that split: a softmax concentrated on one token per
    sequence, a uniform softmax over 32768 tokens, V spanning e4m3's whole range
    (subnormals to 448), queries with x100 outlier dimensions, and scores within 1e-3 of
    each other. Each must stay within the bf16 tolerance of the float64 oracle; the worst
    error / tolerance is printed."""
    H, KVH, D, BS = 32, 8, 128, 256
    g = torch.Generator().manual_seed(["peaked", "uniform_32k", "wide_v", "outlier_q", "tiny_scores"].index(case) + 71)
    lens = [32768] * 2 if case == "uniform_32k" else [int(x) for x in torch.randint(200, 3000, (6,), generator=g)]
    B = len(lens)
    need = [(n + BS - 1) // BS for n in lens]
    NB = sum(need)
    bt = torch.full((B, max(need)), -1, dtype=torch.int32)
    perm = torch.randperm(NB, generator=g)
    pos = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[pos:pos + k].int()
        pos += k
    q = torch.randn(B, H, D, generator=g)
    ks, vs = 0.02, 0.03
    kfill = lambda x: x * 40
    vfill = lambda x: x * 40
    scale = 1.0 / math.sqrt(D)
    if case == "wide_v":
        vfill = lambda x: torch.sign(x) * (2.0 ** (x.abs() * 6 - 9)).clamp(max=448)
    if case == "outlier_q":
        q[:, :, ::16] *= 100.0
    if case == "uniform_32k":
        scale = 1e-6
    if case == "tiny_scores":
        scale = 1e-4
    kc = _fp8_cache(NB * BS, KVH, D, g, kfill).view(NB, BS, KVH, D)
    vc = _fp8_cache(NB * BS, KVH, D, g, vfill).view(NB, BS, KVH, D)
    if case == "peaked":  # one token per sequence aligned with every query head
        for b in range(B):
            t = int(torch.randint(0, lens[b], (1,), generator=g))
            page, off = int(bt[b, t // BS]), t % BS
            for h in range(KVH):
                kc[page, off, h] = (q[b, h * (H // KVH)] * 40).clamp(-448, 448).to(torch.float8_e4m3fn)
    q = q.to(torch.bfloat16)
    cl = torch.tensor(lens, dtype=torch.int64)
    kst, vst = torch.tensor([ks]), torch.tensor([vs])
    ref = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS, k_scale=kst, v_scale=vst)
    out = attn.paged_attention_decode_quantized(
        q.cuda(), kc.cuda(), vc.cuda(), kst.cuda(), vst.cuda(), bt.cuda(), cl.cuda(), scale, H, KVH, D,
        BS, "fp8_per_tensor").cpu()
    atol, rtol = TOL[torch.bfloat16]
    margin = float(((out.double() - ref).abs() / (atol + rtol * ref.abs())).max())
    print(f"\nFP8_ADVERSARIAL {case}: max |err| {float((out.double() - ref).abs().max()):.3e}, "
          f"max |ref| {float(ref.abs().max()):.3e}, worst err/tol {margin:.4f}")
    assert margin <= 1.0
