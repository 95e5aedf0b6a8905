"""KV append on the GPU through the C ABI (Python wrappers) against the CPU oracle:
bf16/fp16/fp32 copies and FP8 E4M3 quantisation must be bit-exact."""
import math

import numpy as np
import pytest
import torch

from conftest import golden, mkv_module
from oracle import fp8_scale_ref, quantize_fp8_ref, store_kvcache_fp8_ref, store_kvcache_ref

pytestmark = pytest.mark.gpu
attn = mkv_module("layers.attention")
lib_mod = mkv_module("_lib")
wl = mkv_module("workloads")


def _case(T, KVH, D, NB, BS, dtype, seed, neg=(), slot_dtype=torch.int64):
    g = torch.Generator().manual_seed(seed)
    key = torch.randn(T, KVH, D, generator=g).to(dtype)
    value = torch.randn(T, KVH, D, generator=g).to(dtype)
    slots = torch.randperm(NB * BS, generator=g)[:T].to(slot_dtype)
    for i in neg:
        slots[i] = -1
    kc = torch.randn(NB, BS, KVH, D, generator=g).to(dtype)
    vc = torch.randn(NB, BS, KVH, D, generator=g).to(dtype)
    return key, value, slots, kc, vc


def _bits(t):
    return t.view(torch.uint8) if t.element_size() == 1 else t.view(torch.int16 if t.element_size() == 2 else torch.int32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D,BS", [(128, 16), (128, 256), (64, 1), (40, 8), (20, 4)])
@pytest.mark.parametrize("slot_dtype", [torch.int64, torch.int32])
def test_store_kvcache_bit_exact(dtype, D, BS, slot_dtype):
    NB = max(40, (77 + BS - 1) // BS + 3)
    key, value, slots, kc, vc = _case(77, 4, D, NB, BS, dtype, 1, neg=(0, 5, 76), slot_dtype=slot_dtype)
    ek, ev = kc.clone(), vc.clone()
    store_kvcache_ref(key, value, ek, ev, slots, BS)
    dk, dv = kc.cuda(), vc.cuda()
    attn.store_kvcache(key.cuda(), value.cuda(), dk, dv, slots.cuda(), BS)
    assert torch.equal(_bits(dk.cpu()), _bits(ek)) and torch.equal(_bits(dv.cpu()), _bits(ev))


def test_store_kvcache_strided_source():
    """K/V as column slices of a fused qkv projection (token stride != KVH*D)."""
    T, H, KVH, D, BS, NB = 50, 8, 2, 128, 16, 8
    qkv = torch.randn(T, (H + 2 * KVH) * D, dtype=torch.bfloat16, device="cuda")
    k = qkv[:, H * D:(H + KVH) * D].view(T, KVH, D)
    v = qkv[:, (H + KVH) * D:].view(T, KVH, D)
    assert not k.is_contiguous()
    slots = torch.randperm(NB * BS)[:T].cuda()
    kc = torch.zeros(NB, BS, KVH, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    attn.store_kvcache(k, v, kc, vc, slots, BS)
    ek, ev = torch.zeros_like(kc).cpu(), torch.zeros_like(vc).cpu()
    store_kvcache_ref(k.cpu(), v.cpu(), ek, ev, slots.cpu(), BS)
    assert torch.equal(kc.cpu().view(torch.int16), ek.view(torch.int16))
    assert torch.equal(vc.cpu().view(torch.int16), ev.view(torch.int16))


def test_out_of_range_slots_are_skipped_and_counted():
    lib = lib_mod.load()
    T, KVH, D, NB, BS = 6, 2, 128, 4, 16
    key = torch.randn(T, KVH, D, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(NB, BS, KVH, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, NB * BS, 5, 10 ** 9, -1, 63], dtype=torch.int64, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = lib.mkv_store_kvcache(key.data_ptr(), key.data_ptr(), KVH * D, D, KVH * D, D,
                               kc.data_ptr(), vc.data_ptr(), NB, BS, slots.data_ptr(), 1, T, KVH,
                               D, lib_mod.DTYPE_BF16, counter.data_ptr(),
                               torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert int(counter) == 2
    flat = kc.view(-1, KVH, D)
    assert torch.equal(flat[0], key[0]) and torch.equal(flat[5], key[2]) and torch.equal(flat[63], key[5])
    assert int((flat.float().abs().sum(dim=(1, 2)) != 0).sum()) == 3


def test_golden_append_bf16_through_cuda():
    g = golden("append_bf16")
    b = lambda a: torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)
    kc, vc = b(g["k_cache_in"]).cuda(), b(g["v_cache_in"]).cuda()
    attn.store_kvcache(b(g["key"]).cuda(), b(g["value"]).cuda(), kc, vc,
                       torch.from_numpy(g["slot_mapping"]).cuda(), int(g["block_size"]))
    assert np.array_equal(kc.cpu().view(torch.int16).numpy().astype(np.uint16), g["k_cache_out"])
    assert np.array_equal(vc.cpu().view(torch.int16).numpy().astype(np.uint16), g["v_cache_out"])


def test_config2_append_bf16_bit_exact():
    w = wl.config2(seed=3)
    KVH, D = w.key.shape[1:]
    kc = torch.zeros(w.num_blocks, w.block_size, KVH, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    attn.store_kvcache(w.key, w.value, kc, vc, w.slot_mapping, w.block_size)
    ek, ev = torch.zeros_like(kc).cpu(), torch.zeros_like(vc).cpu()
    store_kvcache_ref(w.key.cpu(), w.value.cpu(), ek, ev, w.slot_mapping.cpu(), w.block_size)
    assert torch.equal(kc.cpu().view(torch.int16), ek.view(torch.int16))
    assert torch.equal(vc.cpu().view(torch.int16), ev.view(torch.int16))


# ------------------------------------------------------------------------------ FP8
def _torch_cuda_scale(x):
    """The reference's own expression (attention.py:319-320) evaluated by torch on CUDA."""
    return float((x.abs().amax().clamp(min=1e-8) / 448.0).item())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("mag", [1.0, 37.0, 1e-3, 0.0])
def test_fp8_calibration_matches_torch_cuda(dtype, mag):
    T, KVH, D, NB, BS = 300, 8, 128, 64, 16
    for seed in range(4):
        g = torch.Generator().manual_seed(seed)
        key = (torch.randn(T, KVH, D, generator=g) * mag).to(dtype).cuda()
        value = (torch.rand(T, KVH, D, generator=g) * mag * 3).to(dtype).cuda()
        slots = torch.randperm(NB * BS, generator=g)[:T].cuda()
        kc = torch.zeros(NB, BS, KVH, D, dtype=torch.float8_e4m3fn, device="cuda")
        vc = torch.zeros_like(kc)
        ks = torch.ones(1, device="cuda")
        vs = torch.ones(1, device="cuda")
        attn.store_kvcache_fp8(key, value, kc, vc, ks, vs, slots, BS, "fp8_per_tensor")
        assert float(ks) == _torch_cuda_scale(key) == fp8_scale_ref(key.cpu())
        assert float(vs) == _torch_cuda_scale(value) == fp8_scale_ref(value.cpu())


def test_fp8_scale_frozen_after_first_calibration():
    T, KVH, D, NB, BS = 64, 2, 128, 16, 16
    kc = torch.zeros(NB, BS, KVH, D, dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.ones(1, device="cuda")
    vs = torch.tensor([0.25], device="cuda")  # already calibrated: must stay
    first = torch.randn(T, KVH, D, dtype=torch.bfloat16, device="cuda")
    attn.store_kvcache_fp8(first, first, kc, vc, ks, vs, torch.arange(T, device="cuda"), BS,
                           "fp8_per_tensor")
    s0 = float(ks)
    assert s0 == fp8_scale_ref(first.cpu()) and float(vs) == 0.25
    bigger = first * 100
    attn.store_kvcache_fp8(bigger, bigger, kc, vc, ks, vs, torch.arange(T, device="cuda"), BS,
                           "fp8_per_tensor")
    assert float(ks) == s0 and float(vs) == 0.25


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [128, 64, 48])
def test_store_kvcache_fp8_bit_exact(dtype, D):
    T, KVH, NB, BS = 200, 4, 32, 16
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, T, KVH, D, generator=g)
    x = torch.where(torch.rand(x.shape, generator=g) < 0.01, x * 20, x).to(dtype)
    slots = torch.randperm(NB * BS, generator=g)[:T]
    slots[[3, 99]] = -1
    kc = torch.zeros(NB, BS, KVH, D, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    ks, vs = torch.ones(1), torch.ones(1)
    store_kvcache_fp8_ref(x[0], x[1], kc, vc, ks, vs, slots, BS)
    dkc, dvc = torch.zeros_like(kc).cuda(), torch.zeros_like(vc).cuda()
    dks, dvs = torch.ones(1, device="cuda"), torch.ones(1, device="cuda")
    attn.store_kvcache_fp8(x[0].cuda(), x[1].cuda(), dkc, dvc, dks, dvs, slots.cuda(), BS,
                           "fp8_per_tensor")
    assert float(dks) == float(ks) and float(dvs) == float(vs)
    assert torch.equal(dkc.cpu().view(torch.uint8), kc.view(torch.uint8))
    assert torch.equal(dvc.cpu().view(torch.uint8), vc.view(torch.uint8))


def test_fp8_quantisation_edge_values():
    """Rounding midpoints, subnormals, saturation, signed zero, inf and NaN (NaN -> -448,
    as Triton's tl.maximum/tl.minimum return the non-NaN operand)."""
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float()
    v = torch.unique(codes[torch.isfinite(codes)])
    mids = (v[1:] + v[:-1]) / 2
    vals = torch.cat([v, mids, torch.nextafter(mids, torch.full_like(mids, 1e9)),
                      torch.nextafter(mids, torch.full_like(mids, -1e9)),
                      torch.tensor([0.0, -0.0, 500.0, -1e6, float("inf"), float("-inf"), float("nan")])])
    D, KVH, BS = 128, 1, 4
    n = (vals.numel() + D - 1) // D * D
    x = torch.zeros(n)
    x[:vals.numel()] = vals
    T = n // D
    key = x.view(T, KVH, D)
    scale = 0.5  # exact: x / 0.5 = 2x
    expect = quantize_fp8_ref(key, scale)
    kc = torch.zeros((T + BS - 1) // BS, BS, KVH, D, dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.tensor([scale], device="cuda")
    attn.store_kvcache_fp8(key.cuda(), key.cuda(), kc, vc, ks, ks.clone(), torch.arange(T, device="cuda"),
                           BS, "fp8_per_tensor")
    got = kc.view(-1, KVH, D)[:T].cpu()
    assert torch.equal(got.view(torch.uint8), expect.view(torch.uint8))


def test_golden_append_fp8_through_cuda():
    g = golden("append_fp8")
    b = lambda a: torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)
    BS = int(g["block_size"])
    shape = g["k_quot0"].shape
    kc = torch.zeros(shape, dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.zeros_like(kc)
    ks, vs = torch.ones(1, device="cuda"), torch.ones(1, device="cuda")
    for call in (0, 1):
        attn.store_kvcache_fp8(b(g[f"key{call}"]).cuda(), b(g[f"value{call}"]).cuda(), kc, vc, ks, vs,
                               torch.from_numpy(g[f"slot_mapping{call}"]).cuda(), BS, "fp8_per_tensor")
        assert float(ks) == float(g[f"k_scale{call}"][0]) and float(vs) == float(g[f"v_scale{call}"][0])
    exp_k = torch.from_numpy(g["k_quot1"]).to(torch.float8_e4m3fn).view(torch.uint8)
    exp_v = torch.from_numpy(g["v_quot1"]).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(kc.cpu().view(torch.uint8), exp_k) and torch.equal(vc.cpu().view(torch.uint8), exp_v)


def test_config2_append_fp8_bit_exact():
    w = wl.config2(seed=5)
    KVH, D = w.key.shape[1:]
    kc = torch.zeros(w.num_blocks, w.block_size, KVH, D, dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.zeros_like(kc)
    ks, vs = torch.ones(1, device="cuda"), torch.ones(1, device="cuda")
    attn.store_kvcache_fp8(w.key, w.value, kc, vc, ks, vs, w.slot_mapping, w.block_size, "fp8_per_tensor")
    ek, ev = torch.zeros_like(kc).cpu(), torch.zeros_like(vc).cpu()
    eks, evs = torch.ones(1), torch.ones(1)
    store_kvcache_fp8_ref(w.key.cpu(), w.value.cpu(), ek, ev, eks, evs, w.slot_mapping.cpu(), w.block_size)
    assert float(ks) == float(eks) and float(vs) == float(evs)
    assert torch.equal(kc.cpu().view(torch.uint8), ek.view(torch.uint8))
    assert torch.equal(vc.cpu().view(torch.uint8), ev.view(torch.uint8))


def test_fp8_capture_warmup_does_not_calibrate():
    """A runner's eager warm-up on dummy inputs inside fp8_calibration_suspended() leaves the
    sentinel scale alone; the graph captured afterwards calibrates on its first replay with
    real K/V, and later replays keep that scale."""
    T, KVH, D, BS, NB = 8, 4, 128, 16, 8
    g = torch.Generator().manual_seed(3)
    kc = torch.zeros(NB, BS, KVH, D, dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.ones(1, dtype=torch.float32, device="cuda")
    vs = torch.ones(1, dtype=torch.float32, device="cuda")
    key = torch.zeros(T, KVH, D, dtype=torch.bfloat16, device="cuda")
    val = torch.zeros_like(key)
    slots = torch.arange(T, dtype=torch.int64, device="cuda")

    def step():
        attn.store_kvcache_fp8(key, val, kc, vc, ks, vs, slots, BS, "fp8_per_tensor")

    key.copy_(torch.randn(T, KVH, D, generator=g).to(torch.bfloat16))  # dummy warm-up data
    with attn.fp8_calibration_suspended():
        step()
    torch.cuda.synchronize()
    assert float(ks) == 1.0 and float(vs) == 1.0
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), attn.fp8_calibration_suspended():
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    torch.cuda.synchronize()
    assert float(ks) == 1.0  # capture runs nothing
    real_k = torch.randn(T, KVH, D, generator=g) * 3.0
    real_v = torch.randn(T, KVH, D, generator=g) * 0.5
    key.copy_(real_k.to(torch.bfloat16))
    val.copy_(real_v.to(torch.bfloat16))
    graph.replay()
    torch.cuda.synchronize()
    want_k = float((key.abs().amax().float() * (1.0 / 448.0)).to(torch.bfloat16))
    want_v = float((val.abs().amax().float() * (1.0 / 448.0)).to(torch.bfloat16))
    assert float(ks) == want_k and float(vs) == want_v
    key.mul_(10)
    graph.replay()
    torch.cuda.synchronize()
    assert float(ks) == want_k  # frozen after the first calibration


# ------------------------------------------------------- one-launch FP8 store (calibrating)
def _fp8_call(lib, fn, key, value, kc, vc, ks, vs, slots, BS, work, invalid=None):
    T, KVH, D = key.shape
    nb = kc.shape[0]
    args = [key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1), value.stride(0),
            value.stride(1), kc.data_ptr(), vc.data_ptr(), ks.data_ptr(), vs.data_ptr(), nb, BS,
            slots.data_ptr(), lib_mod.INDEX_I64 if slots.dtype == torch.int64 else lib_mod.INDEX_I32,
            T, KVH, D, {torch.bfloat16: 2, torch.float16: 1, torch.float32: 0}[key.dtype]]
    if fn == "mkv_store_kvcache_fp8_calibrating":
        args.append(work)
    st = getattr(lib, fn)(*args, invalid.data_ptr() if invalid is not None else None,
                          torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.mkv_last_error()


@pytest.mark.parametrize("T", [3, 4096, 70001])
@pytest.mark.parametrize("sentinel", ["both", "k", "v", "none"])
def test_fp8_one_launch_equals_calibrate_then_store(T, sentinel):
    """mkv_store_kvcache_fp8_calibrating against the two-kernel sequence
    mkv_calibrate_fp8_scales + mkv_store_kvcache_fp8, byte for byte and scale for scale:
    a few tokens, config 2's 4096 (one wave), and 70001 (grid-stride loops), with either,
    both or neither scale still at the sentinel; slots -1 and out of range included. The
    calibration words are left at zero."""
    lib = lib_mod.load()
    KVH, D, BS = 8, 128, 256
    NB = (T + 300) // BS + 4
    g = torch.Generator().manual_seed(T)
    key = (torch.randn(T, KVH, D, generator=g) * 3).to(torch.bfloat16).cuda()
    value = (torch.randn(T, KVH, D, generator=g) * 0.5).to(torch.bfloat16).cuda()
    slots = torch.randperm(NB * BS, generator=g)[:T]
    slots[::97] = -1
    slots[1::131] = NB * BS + 5  # out of range: skipped and counted
    slots = slots.cuda()
    init = {"both": (1.0, 1.0), "k": (1.0, 0.02), "v": (0.03, 1.0), "none": (0.05, 0.04)}[sentinel]
    outs = []
    for fn in ("two_kernels", "mkv_store_kvcache_fp8_calibrating"):
        kc = torch.zeros(NB, BS, KVH, D, dtype=torch.float8_e4m3fn, device="cuda")
        vc = torch.zeros_like(kc)
        ks = torch.tensor([init[0]], device="cuda")
        vs = torch.tensor([init[1]], device="cuda")
        work = torch.zeros(lib_mod.FP8_CALIB_WORK_BYTES, dtype=torch.uint8, device="cuda")
        inv = torch.zeros(1, dtype=torch.int32, device="cuda")
        if fn == "two_kernels":
            st = lib.mkv_calibrate_fp8_scales(key.data_ptr(), value.data_ptr(), key.stride(0),
                                              key.stride(1), value.stride(0), value.stride(1), T,
                                              KVH, D, 2, ks.data_ptr(), vs.data_ptr(),
                                              work.data_ptr(), torch.cuda.current_stream().cuda_stream)
            assert st == 0
            _fp8_call(lib, "mkv_store_kvcache_fp8", key, value, kc, vc, ks, vs, slots, BS, None, inv)
        else:
            _fp8_call(lib, fn, key, value, kc, vc, ks, vs, slots, BS, work.data_ptr(), inv)
        torch.cuda.synchronize()
        assert int(work.count_nonzero()) == 0
        outs.append((kc.view(torch.uint8).cpu(), vc.view(torch.uint8).cpu(), float(ks), float(vs),
                     int(inv)))
    (k0, v0, ks0, vs0, i0), (k1, v1, ks1, vs1, i1) = outs
    assert (ks0, vs0) == (ks1, vs1)
    if sentinel in ("both", "k"):
        assert ks1 == fp8_scale_ref(key.cpu())
    if sentinel in ("both", "v"):
        assert vs1 == fp8_scale_ref(value.cpu())
    assert torch.equal(k0, k1) and torch.equal(v0, v1)
    assert i0 == i1 == len(range(1, T, 131))
    # and both equal the oracle
    ek = torch.zeros(NB, BS, KVH, D, dtype=torch.float8_e4m3fn)
    ev = torch.zeros_like(ek)
    sl = slots.cpu().clone()
    sl[sl >= NB * BS] = -1
    store_kvcache_fp8_ref(key.cpu(), value.cpu(), ek, ev, torch.tensor([ks1]), torch.tensor([vs1]), sl, BS)
    assert torch.equal(k1, ek.view(torch.uint8)) and torch.equal(v1, ev.view(torch.uint8))


def _e4m3_midpoints():
    """Every rounding midpoint between consecutive finite e4m3 magnitudes (0 .. 448)."""
    vals = sorted(set(torch.arange(0, 0x7F, dtype=torch.uint8).view(torch.float8_e4m3fn).float().tolist()))
    return torch.tensor([(a + b) / 2 for a, b in zip(vals, vals[1:])], dtype=torch.float64)


def _scales_for_midpoint_test():
    g = torch.Generator().manual_seed(77)
    rnd = (torch.rand(24, generator=g, dtype=torch.float64) * 12 - 9).exp2()  # 2^-9 .. 2^3
    s = rnd.float().tolist()
    s += rnd.to(torch.bfloat16).float().tolist()  # calibrated scales are bf16 values
    s += [2.0 ** k for k in (-7, -3, 0, 2)]
    s += [float(torch.tensor(1.0 - 2.0 ** -24, dtype=torch.float32)) * 2.0 ** k for k in (-6, 0, 1)]
    s += [float(torch.tensor(1.0 + 2.0 ** -23, dtype=torch.float32)) * 2.0 ** k for k in (-4, 0)]
    s += [0.1865234375, 0.169921875, 3.0e-3, 7.0 / 3.0]
    return s


@pytest.mark.parametrize("key_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fp8_quantiser_at_rounding_midpoints(key_dtype):
    """The quantiser's quotient x / scale is correctly rounded where it matters: for many
    scales, inputs whose quotients fall on or within three ulp of every e4m3 rounding
    midpoint (float32 keys), and every finite bf16 / fp16 value (16-bit keys), with both
    signs, zeros, infinities and NaN, give the oracle's bytes (IEEE division)."""
    mids = _e4m3_midpoints()
    for s in _scales_for_midpoint_test():
        if key_dtype == torch.float32:
            base = (torch.cat([mids, -mids]) * s).float()
            xs = [base]
            lo = hi = base
            for _ in range(3):
                lo = torch.nextafter(lo, torch.full_like(lo, -math.inf))
                hi = torch.nextafter(hi, torch.full_like(hi, math.inf))
                xs += [lo, hi]
            x = torch.cat(xs + [torch.tensor([0.0, -0.0, math.inf, -math.inf, math.nan, 1e-30, -1e30])])
        else:
            bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16)
            x = bits.view(key_dtype).float()
        n = x.numel()
        T = (n + 15) // 16
        x = torch.cat([x, torch.zeros(T * 16 - n)]).to(key_dtype).view(T, 1, 16)
        slots = torch.arange(T, dtype=torch.int64)
        kc = torch.zeros(T, 1, 1, 16, dtype=torch.float8_e4m3fn, device="cuda")
        vc = torch.zeros_like(kc)
        sc = torch.tensor([s], dtype=torch.float32, device="cuda")
        with attn.fp8_calibration_suspended():  # a scale of exactly 1.0 is not recalibrated
            attn.store_kvcache_fp8(x.cuda(), x.cuda(), kc, vc, sc, sc.clone(), slots.cuda(), 1,
                                   "fp8_per_tensor")
        want = quantize_fp8_ref(x.float(), float(sc)).view(torch.uint8)
        got = kc.cpu().view(torch.uint8).view(T, 1, 16)
        bad = got != want
        assert not bad.any(), (s, x.float()[bad][:5].tolist(), got[bad][:5].tolist(), want[bad][:5].tolist())
