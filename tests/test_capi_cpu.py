"""C-ABI checks that need no GPU: libmkv.so loads, exports every symbol include/mkv.h
declares, and its host-side logic (split planning, workspace sizing, argument
validation) behaves; no call here reaches a CUDA API."""
import ctypes
import os
import re

import pytest

from conftest import REPO, mkv_module

lib_mod = mkv_module("_lib")


def declared_symbols():
    text = open(os.path.join(REPO, "include", "mkv.h")).read()
    return re.findall(r"MKV_API\s+[\w\s\*]+?\b(mkv_\w+)\s*\(", text)


def test_header_and_binding_agree():
    assert sorted(declared_symbols()) == sorted(lib_mod.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(lib_mod.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_header_constants_match_binding():
    text = open(os.path.join(REPO, "include", "mkv.h")).read()
    consts = dict(re.findall(r"#define (MKV_\w+) (\d+)", text))
    assert int(consts["MKV_DTYPE_F32"]) == lib_mod.DTYPE_F32
    assert int(consts["MKV_DTYPE_F16"]) == lib_mod.DTYPE_F16
    assert int(consts["MKV_DTYPE_BF16"]) == lib_mod.DTYPE_BF16
    assert int(consts["MKV_DTYPE_FP8_E4M3"]) == lib_mod.DTYPE_FP8_E4M3
    assert int(consts["MKV_INDEX_I64"]) == lib_mod.INDEX_I64
    assert int(consts["MKV_FP8_CALIB_WORK_BYTES"]) == lib_mod.FP8_CALIB_WORK_BYTES
    assert int(consts["MKV_ERR_WORKSPACE"]) == lib_mod.ERR_WORKSPACE


def test_version_and_status_strings():
    lib = lib_mod.load()
    assert re.fullmatch(rb"\d+\.\d+\.\d+", lib.mkv_version())
    assert lib.mkv_status_string(0) == b"MKV_OK"
    assert lib.mkv_status_string(3) == b"MKV_ERR_WORKSPACE"


@pytest.mark.parametrize("B,H,KVH,BS,MAXB,expect", [
    (256, 32, 8, 256, 32, 0),     # config 3: balanced schedule (0 = chosen on the device)
    (64, 32, 8, 256, 128, 0),     # config 4
    (4, 16, 8, 16, 32, 0),        # config 1
    (1, 8, 8, 16, 1, 0),          # tiny
    (65535, 65535, 65535, 256, 1 << 22, 128),  # work-item bound exceeded: fixed plan
])
def test_split_plan(B, H, KVH, BS, MAXB, expect):
    lib = lib_mod.load()
    assert lib.mkv_paged_decode_num_splits(B, H, KVH, 128, BS, MAXB) == expect


RESIDENT = 148 * 4  # balanced schedule: at most 4 CTAs per SM on 148 SMs


def test_workspace_bytes_balanced():
    """Auto (num_splits = 0): 2 partial slots per resident CTA, heads_per_cta heads each,
    plus one arrival counter per (seq, kv head)."""
    lib = lib_mod.load()
    n = 2 * RESIDENT * 4                   # slots x heads per CTA (group of 4)
    acc = (n * 128 * 4 + 255) // 256 * 256
    ml = (n * 8 + 255) // 256 * 256
    ctr = (256 * 8 * 4 + 255) // 256 * 256
    assert lib.mkv_paged_decode_workspace_bytes(256, 32, 8, 128, 256, 32, 0) == acc + ml + ctr
    # independent of the context length: the same bound serves any table width
    assert lib.mkv_paged_decode_workspace_bytes(256, 32, 8, 128, 256, 4096, 0) == acc + ml + ctr
    # group of 32 query heads -> two head groups of 16
    n16 = 2 * RESIDENT * 16
    ctr16 = (4 * 2 * 2 * 4 + 255) // 256 * 256
    assert lib.mkv_paged_decode_workspace_bytes(4, 64, 2, 128, 16, 8, 0) == \
        (n16 * 128 * 4 + 255) // 256 * 256 + (n16 * 8 + 255) // 256 * 256 + ctr16


def test_prefill_workspace_bytes():
    """The prefill scratch (8-bit pages converted to 16 bits once per call): two 16-bit
    copies of num_seqs x max_num_blocks pages for long chunks of an 8-bit cache, else 0."""
    f = lib_mod.load().mkv_paged_prefill_workspace_bytes
    BF16, F16, F32 = lib_mod.DTYPE_BF16, lib_mod.DTYPE_F16, lib_mod.DTYPE_F32
    FP8, INT8 = lib_mod.DTYPE_FP8_E4M3, lib_mod.DTYPE_INT8
    full = 2 * 8 * 24 * 256 * 8 * 128 * 2
    assert f(8, 8 * 2048, 32, 8, 128, 256, 24, BF16, FP8) == full
    assert f(8, 8 * 2048, 32, 8, 128, 256, 24, F16, INT8) == full
    assert f(8, 8 * 2048, 32, 8, 128, 256, 24, BF16, BF16) == 0      # 16-bit cache
    assert f(8, 8 * 2048, 32, 8, 128, 256, 24, F32, FP8) == 0        # fp32 queries
    assert f(8, 8 * 2048, 32, 8, 64, 256, 24, BF16, FP8) == 0        # head_dim 64
    assert f(8, 8 * 100, 32, 8, 128, 256, 24, BF16, FP8) == 0        # 400 rows per sequence
    assert f(8, 8 * 128, 32, 8, 128, 256, 24, BF16, FP8) == full     # 512 rows per sequence
    assert f(64, 64 * 2048, 32, 8, 128, 256, 128, BF16, FP8) == 0    # 4 GiB: above the 1 GiB cap
    assert f(8, 8 * 2048, 32, 8, 128, 48, 24, BF16, FP8) == 0        # block size not a power of two


def test_workspace_bytes_fixed_splits():
    lib = lib_mod.load()
    n = 256 * 32 * 8                      # (seq, head, split) partials
    acc = (n * 128 * 4 + 255) // 256 * 256
    ml = (n * 8 + 255) // 256 * 256
    ctr = (256 * 8 * 4 + 255) // 256 * 256
    assert lib.mkv_paged_decode_workspace_bytes(256, 32, 8, 128, 256, 32, 8) == acc + ml + ctr
    assert lib.mkv_paged_decode_workspace_bytes(8, 8, 8, 128, 16, 1, 1) == 0   # one split: none
    assert lib.mkv_paged_decode_workspace_bytes(2, 4, 2, 64, 16, 64, 4) > 0


def _decode_call(lib, **kw):
    a = dict(q=1 << 20, qsb=4096, qsh=128, qdt=2, k=1 << 21, v=1 << 22, cdt=2, nb=10, bs=16,
             bt=1 << 23, btt=0, btsb=4, maxb=4, cl=1 << 24, clt=1, B=2, H=8, KVH=2, D=128,
             scale=0.1, out=1 << 25, osb=1024, osh=128, ws=None, wsb=0, ns=0)
    a.update(kw)
    return lib.mkv_paged_decode(a["q"], a["qsb"], a["qsh"], a["qdt"], a["k"], a["v"], a["cdt"],
                                a["nb"], a["bs"], a["bt"], a["btt"], a["btsb"], a["maxb"],
                                a["cl"], a["clt"], a["B"], a["H"], a["KVH"], a["D"], a["scale"],
                                a["out"], a["osb"], a["osh"], a["ws"], a["wsb"], a["ns"], None, None)


@pytest.mark.parametrize("kw,status,msg", [
    (dict(H=7), 1, b"multiple of num_kv_heads"),
    (dict(D=100), 2, b"head_dim"),
    (dict(D=512), 2, b"head_dim"),
    (dict(cdt=3), 1, b"mkv_paged_decode_fp8"),
    (dict(cdt=1), 2, b"cache dtype"),
    (dict(btt=7), 1, b"block_table_index_type"),
    (dict(k=(1 << 21) + 8), 1, b"16-byte aligned"),
    (dict(maxb=64, ns=0, B=512), 3, b"workspace"),
    (dict(maxb=64, ns=8, B=512), 3, b"workspace"),
    (dict(q=None), 1, b"null pointer"),
    (dict(bs=0), 1, b"bad sizes"),
])
def test_decode_argument_validation(kw, status, msg):
    lib = lib_mod.load()
    assert _decode_call(lib, **kw) == status
    assert msg in lib.mkv_last_error()


def test_decode_empty_batch_is_noop():
    lib = lib_mod.load()
    assert _decode_call(lib, B=0, q=None, out=None) == 0


def test_fp8_decode_requires_scales():
    lib = lib_mod.load()
    st = lib.mkv_paged_decode_fp8(1 << 20, 4096, 128, 2, 1 << 21, 1 << 22, None, None, 10, 16,
                                  1 << 23, 0, 4, 4, 1 << 24, 1, 2, 8, 2, 128, 0.1, 1 << 25, 1024,
                                  128, None, 0, 0, None, None)
    assert st == 1 and b"k_scale" in lib.mkv_last_error()


def test_store_argument_validation():
    lib = lib_mod.load()
    st = lib.mkv_store_kvcache(1 << 20, 1 << 21, 256, 128, 256, 128, 1 << 22, 1 << 23, 10, 16,
                               1 << 24, 5, 4, 2, 128, 2, None, None)
    assert st == 1 and b"slot_index_type" in lib.mkv_last_error()
    st = lib.mkv_store_kvcache(1 << 20, 1 << 21, 256, 128, 256, 128, 1 << 22, 1 << 23, 10, 16,
                               1 << 24, 1, 4, 2, 128, 9, None, None)
    assert st == 2 and b"dtype" in lib.mkv_last_error()
    assert lib.mkv_store_kvcache(None, None, 0, 0, 0, 0, None, None, 10, 16, None, 1, 0, 2, 128,
                                 2, None, None) == 0  # zero tokens: nothing to do
    st = lib.mkv_store_kvcache_fp8(1 << 20, 1 << 21, 256, 128, 256, 128, 1 << 22, 1 << 23,
                                   1 << 24, 1 << 25, 10, 16, 1 << 26, 1, 4, 2, 40, 2, None, None)
    assert st == 2 and b"multiple of 16" in lib.mkv_last_error()
    st = lib.mkv_calibrate_fp8_scales(1 << 20, 1 << 21, 256, 128, 256, 128, 4, 2, 128, 3,
                                      1 << 22, 1 << 23, 1 << 24, None)
    assert st == 2 and b"f32, f16 or bf16" in lib.mkv_last_error()
    st = lib.mkv_calibrate_fp8_scales(1 << 20, 1 << 21, 256, 128, 256, 128, 4, 2, 128, 2,
                                      1 << 22, 1 << 23, (1 << 24) + 4, None)
    assert st == 1 and b"8-byte aligned" in lib.mkv_last_error()


def test_python_wrappers_reject_cpu_tensors(attn):
    import torch
    key = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    cache = torch.zeros(8, 16, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        attn.store_kvcache(key, key, cache, cache.clone(), torch.zeros(4, dtype=torch.long), 16)
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        attn.paged_attention_decode(q, cache, cache, torch.zeros(2, 4, dtype=torch.int32),
                                    torch.ones(2, dtype=torch.long), 0.1, 8, 2, 128, 16)
    with pytest.raises(NotImplementedError):
        attn.paged_attention_decode_quantized(q, cache, cache, None, None, None, None, 0.1, 8, 2,
                                              128, 16, "kivi_2bit")
    with pytest.raises(ValueError, match="int8"):  # per-(token, head) INT8 needs int8 pages
        attn.paged_attention_decode_quantized(q, cache, cache, None, None, None, None, 0.1, 8, 2,
                                              128, 16, "int8_per_token_head")
