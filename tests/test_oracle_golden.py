"""Pins the CPU oracle to the reference's own outputs (tests/golden/*.npz, made by
tests/golden/make_golden.py from heart1128/mini-kvllm's functions)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import (
    allreduce_residual_rmsnorm_ref,decode_torch_optimized, e4m3_encode_reference, fp8_scale_ref,
                    paged_decode_ref, paged_prefill_ref, per_token_head_scales_ref,
                    quantize_fp8_ref,
                    store_kvcache_fp8_ref, store_kvcache_quant_per_token_head_ref,
                    store_kvcache_ref)


def bf16(a):
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)


def test_append_bf16_matches_reference():
    g = golden("append_bf16")
    kc, vc = bf16(g["k_cache_in"]).clone(), bf16(g["v_cache_in"]).clone()
    store_kvcache_ref(bf16(g["key"]), bf16(g["value"]), kc, vc, torch.from_numpy(g["slot_mapping"]),
                      int(g["block_size"]))
    assert torch.equal(kc.view(torch.int16), bf16(g["k_cache_out"]).view(torch.int16))
    assert torch.equal(vc.view(torch.int16), bf16(g["v_cache_out"]).view(torch.int16))


def test_fp8_calibration_matches_reference():
    g = golden("append_fp8")
    # first call calibrates from the batch; the second keeps the frozen scale
    assert fp8_scale_ref(bf16(g["key0"])) == float(g["k_scale0"][0])
    assert fp8_scale_ref(bf16(g["value0"])) == float(g["v_scale0"][0])
    assert float(g["k_scale1"][0]) == float(g["k_scale0"][0])
    assert float(g["v_scale1"][0]) == float(g["v_scale0"][0])


@pytest.mark.parametrize("call", [0, 1])
def test_fp8_quotients_match_reference(call):
    """The reference kernel's clamp(x / scale) (captured in fp32 caches) equals the
    oracle's pre-cast quotient at every written slot."""
    g = golden("append_fp8")
    slots = torch.from_numpy(g[f"slot_mapping{call}"])
    keep = slots != -1
    for name, scale_key, quot in (("key", "k_scale", "k_quot"), ("value", "v_scale", "v_quot")):
        x = bf16(g[f"{name}{call}"])
        s = float(g[f"{scale_key}{call}"][0])
        q = x.float() / torch.tensor(s, dtype=torch.float32)
        q = q.clamp(-448.0, 448.0)
        ref = torch.from_numpy(g[f"{quot}{call}"]).view(-1, x.shape[1], x.shape[2])[slots[keep]]
        assert torch.equal(q[keep], ref)
        # and the e4m3 bytes of those quotients are the oracle's quantisation
        assert torch.equal(quantize_fp8_ref(x, s)[keep].view(torch.uint8),
                           ref.to(torch.float8_e4m3fn).view(torch.uint8))


def test_fp8_append_end_to_end_matches_reference():
    g = golden("append_fp8")
    BS = int(g["block_size"])
    shape = g["k_quot0"].shape
    kc = torch.zeros(shape, dtype=torch.float8_e4m3fn)
    vc = torch.zeros(shape, dtype=torch.float8_e4m3fn)
    ks, vs = torch.ones(1), torch.ones(1)
    for call in (0, 1):
        store_kvcache_fp8_ref(bf16(g[f"key{call}"]), bf16(g[f"value{call}"]), kc, vc, ks, vs,
                              torch.from_numpy(g[f"slot_mapping{call}"]), BS)
        assert float(ks[0]) == float(g[f"k_scale{call}"][0])
        assert float(vs[0]) == float(g[f"v_scale{call}"][0])
    exp_k = torch.from_numpy(g["k_quot1"]).to(torch.float8_e4m3fn)
    exp_v = torch.from_numpy(g["v_quot1"]).to(torch.float8_e4m3fn)
    assert torch.equal(kc.view(torch.uint8), exp_k.view(torch.uint8))
    assert torch.equal(vc.view(torch.uint8), exp_v.view(torch.uint8))


def test_e4m3_cast_pinned_by_independent_encoder():
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(200_000) * s for s in (1e-3, 0.1, 1, 50, 300)])
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    v = np.unique(codes[np.isfinite(codes)])
    mids = (v[1:] + v[:-1]) / 2
    x = np.clip(np.concatenate([x, mids, v, [0.0, -0.0]]), -448, 448).astype(np.float32)
    t = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(t, e4m3_encode_reference(x))


def _decode_inputs(g, fp8=False):
    H, KVH = int(g["num_heads"]), int(g["num_kv_heads"])
    q = torch.from_numpy(g["query"])
    if fp8:
        kc = torch.from_numpy(g["k_cache_e4m3"]).view(torch.float8_e4m3fn)
        vc = torch.from_numpy(g["v_cache_e4m3"]).view(torch.float8_e4m3fn)
    else:
        kc, vc = torch.from_numpy(g["k_cache"]), torch.from_numpy(g["v_cache"])
    return q, kc, vc, torch.from_numpy(g["block_tables"]), torch.from_numpy(g["context_lens"]), \
        float(g["scale"]), H, KVH, q.shape[2], int(g["block_size"])


def test_decode_oracle_matches_reference_kernel():
    g = golden("decode_small")
    args = _decode_inputs(g)
    out = paged_decode_ref(*args)
    ref = torch.from_numpy(g["out"]).double()
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(out), nan)  # context 0 -> NaN in both
    assert torch.allclose(out[~nan], ref[~nan], atol=2e-6, rtol=1e-5)


def test_decode_fp8_oracle_matches_reference_kernel():
    g = golden("decode_fp8")
    q, kc, vc, bt, cl, scale, H, KVH, D, BS = _decode_inputs(g, fp8=True)
    out = paged_decode_ref(q, kc, vc, bt, cl, scale, H, KVH, D, BS,
                           k_scale=torch.from_numpy(g["k_scale"]), v_scale=torch.from_numpy(g["v_scale"]))
    assert torch.allclose(out, torch.from_numpy(g["out"]).double(), atol=2e-6, rtol=1e-5)


def test_decode_config1_oracles_match_reference():
    from golden.make_golden import _sha, config1_inputs
    g = golden("decode_config1")
    inp = config1_inputs(int(g["seed"]))
    assert _sha(inp["query"], inp["k_cache"], inp["v_cache"], inp["block_tables"],
                inp["context_lens"]) == str(g["inputs_sha256"]), "seeded input generation drifted"
    args = (torch.from_numpy(inp["query"]), torch.from_numpy(inp["k_cache"]),
            torch.from_numpy(inp["v_cache"]), torch.from_numpy(inp["block_tables"]),
            torch.from_numpy(inp["context_lens"]), float(g["scale"]), inp["num_heads"],
            inp["num_kv_heads"], inp["head_dim"], inp["block_size"])
    ref = torch.from_numpy(g["out"])
    assert torch.allclose(decode_torch_optimized(*args), ref, atol=1e-6, rtol=1e-6)
    assert torch.allclose(paged_decode_ref(*args).float(), ref, atol=2e-6, rtol=1e-5)


# ------------------------------------------------------------- per-(token, head) modes
def _pth_written(g):
    slots = torch.from_numpy(g["slot_mapping"])
    return slots, slots != -1


def test_fp8_per_token_head_scales_and_quotients_match_reference():
    """Per-row scales (amax / 448, 1.0 for the all-zero row) and the kernel's pre-cast
    clamp(x / scale) equal the oracle's at every written slot; unwritten slots stay."""
    g = golden("append_fp8_pth")
    slots, keep = _pth_written(g)
    for name, sk, qk in (("key", "k_scales", "k_quot"), ("value", "v_scales", "v_quot")):
        x = bf16(g[name])
        T, KVH, D = x.shape
        sc = per_token_head_scales_ref(x, "fp8")
        ref_sc = torch.from_numpy(g[sk]).view(-1, KVH)
        assert torch.equal(sc[keep], ref_sc[slots[keep]])
        assert int((ref_sc == -1.0).all(dim=1).sum()) == ref_sc.shape[0] - int(keep.sum())
        assert float(sc[5, 1]) == 1.0  # all-zero row
        quot = (x.float() / sc.unsqueeze(-1)).clamp(-448.0, 448.0)
        ref_q = torch.from_numpy(g[qk]).view(-1, KVH, D)[slots[keep]]
        assert torch.equal(quot[keep], ref_q)


def test_fp8_per_token_head_store_end_to_end():
    g = golden("append_fp8_pth")
    slots, keep = _pth_written(g)
    shape = g["k_quot"].shape
    kc = torch.zeros(shape, dtype=torch.float8_e4m3fn)
    vc = torch.zeros(shape, dtype=torch.float8_e4m3fn)
    ks = torch.full(shape[:3], -1.0)
    vs = torch.full(shape[:3], -1.0)
    store_kvcache_quant_per_token_head_ref(bf16(g["key"]), bf16(g["value"]), kc, vc, ks, vs, slots,
                                           int(g["block_size"]), "fp8")
    assert torch.equal(ks, torch.from_numpy(g["k_scales"]))
    assert torch.equal(vs, torch.from_numpy(g["v_scales"]))
    exp_k = torch.from_numpy(g["k_quot"]).to(torch.float8_e4m3fn)
    assert torch.equal(kc.view(torch.uint8), exp_k.view(torch.uint8))


def test_int8_store_matches_reference():
    """INT8 bytes and scales bit-exact, including the all-zero row (scale 1e-6) and a row
    of exact halves rounded away from zero."""
    g = golden("append_int8")
    slots, keep = _pth_written(g)
    kc = torch.zeros(g["k_cache"].shape, dtype=torch.int8)
    vc = torch.zeros_like(kc)
    ks = torch.full(g["k_scales"].shape, -1.0)
    vs = torch.full(g["v_scales"].shape, -1.0)
    store_kvcache_quant_per_token_head_ref(bf16(g["key"]), bf16(g["value"]), kc, vc, ks, vs, slots,
                                           int(g["block_size"]), "int8")
    assert torch.equal(kc, torch.from_numpy(g["k_cache"]))
    assert torch.equal(vc, torch.from_numpy(g["v_cache"]))
    assert torch.equal(ks, torch.from_numpy(g["k_scales"]))
    assert torch.equal(vs, torch.from_numpy(g["v_scales"]))
    x = bf16(g["key"])
    assert float(per_token_head_scales_ref(x, "int8")[5, 1]) == float(np.float32(1e-6))
    row = torch.from_numpy(g["k_cache"]).view(-1, x.shape[1], x.shape[2])[int(slots[9])][0]
    assert row[:4].tolist() == [3, -3, 1, -127]  # 2.5 -> 3, -2.5 -> -3, 0.5 -> 1


@pytest.mark.parametrize("mode", ["fp8", "int8"])
def test_per_token_head_decode_oracle_matches_reference_kernel(mode):
    g = golden(f"decode_{mode}_pth" if mode == "fp8" else "decode_int8")
    H, KVH = int(g["num_heads"]), int(g["num_kv_heads"])
    q = torch.from_numpy(g["query"])
    if mode == "fp8":
        kc = torch.from_numpy(g["k_cache_e4m3"]).view(torch.float8_e4m3fn)
        vc = torch.from_numpy(g["v_cache_e4m3"]).view(torch.float8_e4m3fn)
    else:
        kc, vc = torch.from_numpy(g["k_cache_i8"]), torch.from_numpy(g["v_cache_i8"])
    out = paged_decode_ref(q, kc, vc, torch.from_numpy(g["block_tables"]),
                           torch.from_numpy(g["context_lens"]), float(g["scale"]), H, KVH,
                           q.shape[2], int(g["block_size"]), k_scales=torch.from_numpy(g["k_scales"]),
                           v_scales=torch.from_numpy(g["v_scales"]))
    assert torch.allclose(out, torch.from_numpy(g["out"]).double(), atol=2e-6, rtol=1e-5)


# ---------------------------------------------------------------------- prefill / extend
@pytest.mark.parametrize("which", ["triton", "torch"])
def test_prefill_oracle_matches_reference(which):
    """Chunked prefill over cached prefixes: the oracle against the reference's Triton kernel
    (with a -1 page inside a context, skipped) and its torch version (all pages valid)."""
    g = golden("prefill")
    bt = torch.from_numpy(g["block_tables"] if which == "triton" else g["block_tables_torch"])
    out = paged_prefill_ref(torch.from_numpy(g["query"]), torch.from_numpy(g["k_cache"]),
                            torch.from_numpy(g["v_cache"]), bt, torch.from_numpy(g["context_lens"]),
                            torch.from_numpy(g["cu_seqlens_q"]), torch.from_numpy(g["positions"]),
                            float(g["scale"]), int(g["num_heads"]), int(g["num_kv_heads"]),
                            int(g["block_size"]))
    ref = torch.from_numpy(g["out"] if which == "triton" else g["out_torch"]).double()
    assert torch.allclose(out, ref, atol=2e-6, rtol=1e-5)


# ------------------------------------------------- all-reduce + residual add + RMSNorm
def test_residual_rmsnorm_oracle_matches_reference():
    """The fused all-reduce + residual + RMSNorm oracle against the reference's
    LayerNorm.residual_rms_forward (run eagerly, in bf16 steps): the all-reduced sum and
    the residual output bit-exact, the normalised output to bf16 accuracy (the reference
    computes it in fp32 on the GPU, under torch.compile)."""
    g = golden("residual_rmsnorm")
    b = lambda k: torch.from_numpy(g[k].astype(np.int16)).view(torch.bfloat16)
    out, s = allreduce_residual_rmsnorm_ref(b("partials"), b("residual"), b("weight"), float(g["eps"]))
    assert torch.equal(b("partials").float().sum(0).bfloat16(), b("x"))
    assert torch.equal(s, b("s"))
    assert torch.allclose(out.float(), b("out").float(), atol=2e-2, rtol=1e-2)


def test_varlen_prefill_oracle_matches_reference():
    """varlen_prefill_ref against flash_attention_prefill (attention.py:446-516) run by
    the Triton interpreter on ragged sequences (lengths 5, 37, 1, 64, 70), fp32."""
    from oracle import varlen_prefill_ref
    g = golden("varlen_prefill")
    out = varlen_prefill_ref(torch.from_numpy(g["query"]), torch.from_numpy(g["key"]),
                             torch.from_numpy(g["value"]), torch.from_numpy(g["cu_seqlens"]),
                             float(g["scale"]), int(g["num_heads"]), int(g["num_kv_heads"]))
    assert torch.allclose(out, torch.from_numpy(g["out"]).double(), atol=2e-6, rtol=1e-5)
