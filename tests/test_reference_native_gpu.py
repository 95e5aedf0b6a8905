"""libmkv against the reference's own GPU path, run natively on the B200.

The reference (heart1128/mini-kvllm, unmodified) is installed into baseline/_ref with
`pip install --target baseline/_ref <reference checkout>`; these tests import its
`myvllm` package from there and skip when that install is absent. Its Triton kernels
then run compiled for the GPU, not under the interpreter that made tests/golden/.

What is compared, on the BASELINE shapes:
  * the bf16 append (store_kvcache, attention.py:67-108): bytes, bit for bit;
  * the FP8 per-tensor append (store_kvcache_fp8, attention.py:281-333): the calibrated
    scales bit for bit, and every quantised byte. A byte may differ only where the
    reference's Triton division (`/` on float32 compiles to the approximate
    div.full.f32, at most 2 ulp from the quotient) lands on the other side of an e4m3
    rounding boundary: each differing byte must be the e4m3 value of a quotient within
    2 ulp of the correctly rounded one. The counts are printed (NATIVE_PARITY lines);
  * the per-(token, head) FP8 / INT8 appends the same way, scales included;
  * the decodes (paged_attention_decode, paged_attention_decode_quantized) within the
    decode tolerance, the worst error / tolerance printed;
  * the drop-in: the reference's own Attention module (attention.py:1617-1807), its
    five hot-path functions replaced by this library's as INTEGRATION.md shows, driven
    over several decode steps by block tables from the reference's BlockManager
    (block_manager.py:80-155) through DecodeMetadataBuilder, against the oracle.
"""
import importlib
import json
import math
import os
import sys

import pytest
import torch

from conftest import REPO, mkv_module
from oracle import (paged_decode_ref, store_kvcache_fp8_ref,
                    store_kvcache_quant_per_token_head_ref, store_kvcache_ref)

pytestmark = pytest.mark.gpu
attn = mkv_module("layers.attention")
wl = mkv_module("workloads")
kvc = mkv_module("engine.kv_cache")

REF_DIR = os.path.join(REPO, "baseline", "_ref")
TOL = (2e-2, 1e-2)  # bf16 outputs, fp32 accumulation (the BASELINE bar)


def _ref(name):
    if not os.path.isdir(os.path.join(REF_DIR, "myvllm")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    return importlib.import_module(name)


@pytest.fixture(scope="module")
def ref_attn():
    return _ref("myvllm.layers.attention")


def report(tag, **kw):
    print(f"\nNATIVE_PARITY {tag} {json.dumps(kw)}")


def e4m3_of(q):
    """Saturating e4m3 bytes of float32 quotients (the clamp of the reference first)."""
    q = torch.where(torch.isnan(q), torch.full_like(q, -448.0), q).clamp(-448.0, 448.0)
    return q.to(torch.float8_e4m3fn).view(torch.uint8)


def quotient_neighbours(q, ulps=2):
    """q and its float32 neighbours up to `ulps` steps either way, stacked on dim 0."""
    out, lo, hi = [q], q, q
    for _ in range(ulps):
        lo = torch.nextafter(lo, torch.full_like(lo, -math.inf))
        hi = torch.nextafter(hi, torch.full_like(hi, math.inf))
        out += [lo, hi]
    return torch.stack(out)


def explained_by_division(x, scale, ref_bytes):
    """Which differing bytes are e4m3(x / scale) for a quotient within 2 ulp of the
    correctly rounded one (scale broadcast against x)."""
    q = x.float() / scale
    cands = e4m3_of(quotient_neighbours(q))
    return (cands == ref_bytes.unsqueeze(0)).any(0)


# ------------------------------------------------------------------ appends (config 2)
def test_native_append_bf16_config2(ref_attn):
    a = wl.config2(seed=0)
    shape = (a.num_blocks, a.block_size, 8, 128)
    ref_k, ref_v = torch.zeros(shape, dtype=torch.bfloat16, device="cuda"), torch.zeros(shape, dtype=torch.bfloat16, device="cuda")
    our_k, our_v = torch.zeros_like(ref_k), torch.zeros_like(ref_v)
    ref_attn.store_kvcache(a.key, a.value, ref_k, ref_v, a.slot_mapping, a.block_size)
    attn.store_kvcache(a.key, a.value, our_k, our_v, a.slot_mapping, a.block_size)
    torch.cuda.synchronize()
    diff = int((ref_k.view(torch.int16) != our_k.view(torch.int16)).sum() +
               (ref_v.view(torch.int16) != our_v.view(torch.int16)).sum())
    report("append_bf16_config2", tokens=a.key.shape[0], differing_bytes=diff)
    assert diff == 0


def test_native_append_fp8_per_tensor_config2(ref_attn):
    """Two appends: the first calibrates both scales from the sentinel 1.0, the second
    (other data) quantises with the frozen scales."""
    a = wl.config2(seed=0)
    b = wl.config2(seed=1)
    shape = (a.num_blocks, a.block_size, 8, 128)
    caches = {k: [torch.zeros(shape, dtype=torch.float8_e4m3fn, device="cuda") for _ in range(2)]
              for k in ("ref", "ours")}
    scales = {k: [torch.ones(1, device="cuda") for _ in range(2)] for k in ("ref", "ours")}
    total = unexplained = 0
    for step, w in enumerate((a, b)):
        rk, rv = caches["ref"]
        ok_, ov = caches["ours"]
        ref_attn.store_kvcache_fp8(w.key, w.value, rk, rv, *scales["ref"], w.slot_mapping,
                                      w.block_size, "fp8_per_tensor")
        attn.store_kvcache_fp8(w.key, w.value, ok_, ov, *scales["ours"], w.slot_mapping,
                               w.block_size, "fp8_per_tensor")
        torch.cuda.synchronize()
        for i in range(2):
            assert float(scales["ref"][i]) == float(scales["ours"][i]), (step, i)
        slots = w.slot_mapping
        for x, rc, oc, sc in ((w.key, rk, ok_, scales["ref"][0]), (w.value, rv, ov, scales["ref"][1])):
            rb = rc.view(-1, 8, 128)[slots].view(torch.uint8)
            ob = oc.view(-1, 8, 128)[slots].view(torch.uint8)
            bad = rb != ob
            total += int(bad.sum())
            if bad.any():
                expl = explained_by_division(x[bad], sc, rb[bad])
                unexplained += int((~expl).sum())
    report("append_fp8_per_tensor_config2", tokens=a.key.shape[0], calls=2,
           scale_k=float(scales["ours"][0]), scale_v=float(scales["ours"][1]),
           differing_bytes=total, of_bytes=4 * a.key.numel(), unexplained=unexplained)
    assert unexplained == 0


@pytest.mark.parametrize("mode", ["fp8_per_token_head", "int8_per_token_head"])
def test_native_append_per_token_head_config2(ref_attn, mode):
    a = wl.config2(seed=2)
    shape = (a.num_blocks, a.block_size, 8, 128)
    cdt = torch.int8 if mode.startswith("int8") else torch.float8_e4m3fn
    mk = lambda: (torch.zeros(shape, dtype=cdt, device="cuda"),
                  torch.ones(shape[:3], dtype=torch.float32, device="cuda"))
    (rk, rks), (rv, rvs), (ok_, oks), (ov, ovs) = mk(), mk(), mk(), mk()
    if mode.startswith("int8"):
        ref_attn.store_kvcache_int8(a.key, a.value, rk, rv, rks, rvs, a.slot_mapping, a.block_size)
        attn.store_kvcache_int8(a.key, a.value, ok_, ov, oks, ovs, a.slot_mapping, a.block_size)
    else:
        ref_attn.store_kvcache_fp8(a.key, a.value, rk, rv, rks, rvs, a.slot_mapping,
                                      a.block_size, mode)
        attn.store_kvcache_fp8(a.key, a.value, ok_, ov, oks, ovs, a.slot_mapping, a.block_size, mode)
    torch.cuda.synchronize()
    slots = a.slot_mapping
    stats = dict(scale_diff=0, scale_max_ulps=0, byte_diff=0, byte_unexplained=0)
    for x, rc, oc, rs, os_ in ((a.key, rk, ok_, rks, oks), (a.value, rv, ov, rvs, ovs)):
        s_ref = rs.view(-1, 8)[slots]
        s_our = os_.view(-1, 8)[slots]
        sd = s_ref != s_our
        stats["scale_diff"] += int(sd.sum())
        if sd.any():  # the reference's amax / qmax is the approximate division
            ulps = (s_ref.view(torch.int32).long() - s_our.view(torch.int32).long()).abs().max()
            stats["scale_max_ulps"] = max(stats["scale_max_ulps"], int(ulps))
        rb = rc.view(-1, 8, 128)[slots].view(torch.uint8)
        ob = oc.view(-1, 8, 128)[slots].view(torch.uint8)
        bad = rb != ob
        stats["byte_diff"] += int(bad.sum())
        if bad.any():
            xs = x.float()[bad]
            sr = s_ref.unsqueeze(-1).expand_as(x)[bad]
            if mode.startswith("int8"):
                # x * (1 / scale) rounded half away from zero: a differing byte is one step
                # away, at a product within 1e-5 (relative) of a rounding boundary
                v = xs * (1.0 / sr)
                frac = (v.abs() - v.abs().floor() - 0.5).abs()
                step = (rb[bad].view(torch.int8).int() - ob[bad].view(torch.int8).int()).abs()
                ok = (step == 1) & (frac <= 1e-5 * v.abs().clamp(min=1.0))
            else:
                ok = explained_by_division(xs, sr, rb[bad])
            stats["byte_unexplained"] += int((~ok).sum())
    report(f"append_{mode}_config2", tokens=a.key.shape[0], of_bytes=2 * a.key.numel(), **stats)
    assert stats["scale_max_ulps"] <= 2
    assert stats["byte_unexplained"] == 0


# ------------------------------------------------------------------ decodes
def _margin(got, ref):
    atol, rtol = TOL
    return float(((got.double() - ref.double()).abs() / (atol + rtol * ref.double().abs())).max())


def test_native_decode_bf16_config3(ref_attn):
    w = wl.config3(seed=1, with_append=False)
    args = (w.query, w.k_cache, w.v_cache, w.block_tables, w.context_lens, w.scale, w.num_heads,
            w.num_kv_heads, w.head_dim, w.block_size)
    ref = ref_attn.paged_attention_decode(*args)
    ours = attn.paged_attention_decode(*args)
    torch.cuda.synchronize()
    m = _margin(ours, ref)
    report("decode_bf16_config3", seqs=w.query.shape[0],
           max_abs_diff=float((ours.float() - ref.float()).abs().max()), worst_err_over_tol=m)
    assert m <= 1.0


def test_native_decode_fp8_config4(ref_attn):
    w = wl.config4(seed=1, with_append=False)
    args = (w.query, w.k_cache, w.v_cache, w.k_scale, w.v_scale, w.block_tables, w.context_lens,
            w.scale, w.num_heads, w.num_kv_heads, w.head_dim, w.block_size, "fp8_per_tensor")
    ref = ref_attn.paged_attention_decode_quantized(*args)
    ours = attn.paged_attention_decode_quantized(*args)
    torch.cuda.synchronize()
    m = _margin(ours, ref)
    report("decode_fp8_config4", seqs=w.query.shape[0],
           max_abs_diff=float((ours.float() - ref.float()).abs().max()), worst_err_over_tol=m)
    assert m <= 1.0


@pytest.mark.parametrize("mode", ["fp8_per_token_head", "int8_per_token_head"])
def test_native_decode_per_token_head(ref_attn, mode):
    """Config 3's heads and pages on 32 sequences; the caches are written by the
    reference's own quantising append, so both decodes read the same bytes and scales."""
    g = torch.Generator().manual_seed(5)
    lens = torch.randint(1024, 8193, (32,), generator=g).tolist()
    w = wl.decode_workload("pth", 32, 32, 8, 128, 256, lens, seed=5, with_append=False)
    cdt = torch.int8 if mode.startswith("int8") else torch.float8_e4m3fn
    NB = w.k_cache.shape[0]
    kc = torch.zeros(NB, 256, 8, 128, dtype=cdt, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.ones(NB, 256, 8, device="cuda")
    vs = torch.ones_like(ks)
    slots = torch.arange(NB * 256, device="cuda")
    src_k = w.k_cache.view(-1, 8, 128)
    src_v = w.v_cache.view(-1, 8, 128)
    if mode.startswith("int8"):
        ref_attn.store_kvcache_int8(src_k, src_v, kc, vc, ks, vs, slots, 256)
    else:
        ref_attn.store_kvcache_fp8(src_k, src_v, kc, vc, ks, vs, slots, 256, mode)
    args = (w.query, kc, vc, ks, vs, w.block_tables, w.context_lens, w.scale, 32, 8, 128, 256, mode)
    ref = ref_attn.paged_attention_decode_quantized(*args)
    ours = attn.paged_attention_decode_quantized(*args)
    torch.cuda.synchronize()
    m = _margin(ours, ref)
    report(f"decode_{mode}", seqs=32, max_abs_diff=float((ours.float() - ref.float()).abs().max()),
           worst_err_over_tol=m)
    assert m <= 1.0


# ------------------------------------------------------------------ drop-in
DROPIN_NAMES = ("store_kvcache", "store_kvcache_int8", "store_kvcache_fp8",
                "paged_attention_decode", "paged_attention_decode_quantized")


@pytest.mark.parametrize("mode", ["auto", "fp8_per_tensor", "fp8_per_token_head", "int8_per_token_head"])
def test_dropin_reference_attention_module(ref_attn, monkeypatch, mode):
    """The reference's Attention.forward with the five functions replaced by this
    library's (the INTEGRATION.md assignments), over prompt appends and six decode
    steps. Block tables come from the reference's BlockManager (allocate, then append
    per step); the per-step metadata from DecodeMetadataBuilder, checked against the
    reference's prepare_decode formulas; outputs against the float64 oracle run on a
    CPU mirror of the cache."""
    rctx = _ref("myvllm.utils.context")
    bm_mod = _ref("myvllm.engine.block_manager")
    seq_mod = _ref("myvllm.engine.sequence")
    for name in DROPIN_NAMES:
        monkeypatch.setattr(ref_attn, name, getattr(attn, name))

    H, KVH, D, BS, NB, B = 16, 4, 128, 16, 96, 6
    g = torch.Generator().manual_seed(7)
    cache = kvc.allocate_kv_cache(1, NB, BS, KVH, D, mode)
    layer = ref_attn.Attention(H, D, scale=1.0, num_kv_heads=KVH, block_size=BS).cuda()
    assert kvc.bind_kv_cache(layer.modules(), cache) == 1
    # CPU mirror of the cache for the oracle
    kc_cpu = torch.zeros(cache.kv.shape[2:], dtype=cache.kv.dtype)
    vc_cpu = torch.zeros_like(kc_cpu)
    if mode == "fp8_per_tensor":
        ks_cpu, vs_cpu = torch.ones(1), torch.ones(1)
    elif mode != "auto":
        ks_cpu, vs_cpu = torch.ones(NB, BS, KVH), torch.ones(NB, BS, KVH)

    def oracle_store(k, v, slots):
        if mode == "auto":
            store_kvcache_ref(k, v, kc_cpu, vc_cpu, slots, BS)
        elif mode == "fp8_per_tensor":
            store_kvcache_fp8_ref(k, v, kc_cpu, vc_cpu, ks_cpu, vs_cpu, slots, BS)
        else:
            store_kvcache_quant_per_token_head_ref(k, v, kc_cpu, vc_cpu, ks_cpu, vs_cpu, slots, BS,
                                                   mode.split("_")[0])

    manager = bm_mod.BlockManager(NB, BS)
    prompts = [int(x) for x in torch.randint(1, 70, (B,), generator=g)]
    seqs = [seq_mod.Sequence(list(range(100 * i, 100 * i + n)), block_size=BS)
            for i, n in enumerate(prompts)]
    builder = kvc.DecodeMetadataBuilder(B, 8, BS)
    for i, s in enumerate(seqs):
        manager.allocate(s)
        builder.set_table(i, s.block_table)
        # the prompt's K/V, appended as the reference's prefill would (slot of each token)
        n = len(s)
        slots = torch.tensor([s.block_table[t // BS] * BS + t % BS for t in range(n)])
        k = torch.randn(n, KVH, D, generator=g).to(torch.bfloat16)
        v = torch.randn(n, KVH, D, generator=g).to(torch.bfloat16)
        k_cache, v_cache, ks, vs = cache.layer(0)
        if mode == "auto":
            ref_attn.store_kvcache(k.cuda(), v.cuda(), k_cache, v_cache, slots.cuda(), BS)
        elif mode == "int8_per_token_head":
            ref_attn.store_kvcache_int8(k.cuda(), v.cuda(), k_cache, v_cache, ks, vs, slots.cuda(), BS)
        else:
            ref_attn.store_kvcache_fp8(k.cuda(), v.cuda(), k_cache, v_cache, ks, vs, slots.cuda(), BS, mode)
        oracle_store(k, v, slots)

    atol, rtol = TOL
    for step in range(6):
        for i, s in enumerate(seqs):  # the scheduler's order: new token, then append
            s.append_token(1000 + step)
            before = len(s.block_table)
            manager.append(s)
            for blk in s.block_table[before:]:  # the block manager took a new block
                builder.append(i, blk)
        md = builder.step(list(range(B)), [len(s) for s in seqs])
        # the reference's prepare_decode formulas (model_runner.py:636-641)
        want_slots = [s.block_table[-1] * BS + s.last_block_num_tokens - 1 for s in seqs]
        assert md.slot_mapping.cpu().tolist() == want_slots
        assert md.context_lens.cpu().tolist() == [len(s) for s in seqs]
        rctx.set_context(is_prefill=False, slot_mapping=md.slot_mapping,
                         context_lens=md.context_lens, block_tables=md.block_tables)
        q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16)
        o = layer(q.cuda(), k.cuda(), v.cuda())
        torch.cuda.synchronize()
        rctx.reset_context()
        oracle_store(k, v, md.slot_mapping.cpu())
        bt = md.block_tables.cpu()
        kw = {}
        if mode == "fp8_per_tensor":
            kw = dict(k_scale=ks_cpu, v_scale=vs_cpu)
        elif mode != "auto":
            kw = dict(k_scales=ks_cpu, v_scales=vs_cpu)
        ref = paged_decode_ref(q, kc_cpu, vc_cpu, bt, md.context_lens.cpu(), 1.0 / math.sqrt(D),
                               H, KVH, D, BS, **kw)
        assert o.shape == (B, H * D)
        assert torch.allclose(o.view(B, H, D).cpu().double(), ref, atol=atol, rtol=rtol), step
    # the device cache holds exactly the oracle's bytes (and scales)
    k_cache, v_cache, ks, vs = cache.layer(0)
    view = torch.int16 if mode == "auto" else torch.uint8
    assert torch.equal(k_cache.cpu().view(view), kc_cpu.view(view))
    assert torch.equal(v_cache.cpu().view(view), vc_cpu.view(view))
    if mode != "auto":
        assert torch.equal(ks.cpu(), ks_cpu) and torch.equal(vs.cpu(), vs_cpu)
