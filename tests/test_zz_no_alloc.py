"""The allocation-free decode entry point, mkv_paged_decode_noalloc.

Some callers of this library cannot allocate device memory themselves (a runtime that
reserves all device memory at start-up, a serving loop that must not pay cudaMalloc's
synchronisation, a cgo/JNI caller without a device allocator), so they cannot create the
split-KV workspace mkv_paged_decode asks for. mkv_paged_decode_noalloc uses scratch
built into the library instead. These tests call both entry points through the C ABI
and require the same result (within the decode tolerances used everywhere in this
suite) on two calls in a row, since the built-in scratch keeps the previous call's
contents. This file is named to be collected last.
"""
import ctypes
import math

import pytest
import torch

from conftest import mkv_module

pytestmark = pytest.mark.gpu
lib_mod = mkv_module("_lib")

DT = {torch.bfloat16: lib_mod.DTYPE_BF16, torch.float16: lib_mod.DTYPE_F16,
      torch.float32: lib_mod.DTYPE_F32}
TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (2e-2, 1e-2), torch.bfloat16: (2e-2, 1e-2)}


def paged_inputs(B, H, KVH, D, BS, lens, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    need = [(n + BS - 1) // BS for n in lens]
    nb = sum(need) + 3
    perm = torch.randperm(nb, generator=g)
    bt = torch.full((B, max(need)), -1, dtype=torch.int32)
    pos = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[pos:pos + k].int()
        pos += k
    q = torch.randn(B, H, D, generator=g).to(dtype).cuda()
    kc = torch.randn(nb, BS, KVH, D, generator=g).to(dtype).cuda()
    vc = torch.randn(nb, BS, KVH, D, generator=g).to(dtype).cuda()
    return q, kc, vc, bt.cuda(), torch.tensor(lens, dtype=torch.int64).cuda()


def common_args(q, kc, vc, bt, cl, H, KVH, D, BS, out):
    nb = kc.shape[0]
    return [q.data_ptr(), q.stride(0), q.stride(1), DT[q.dtype], kc.data_ptr(), vc.data_ptr(),
            DT[kc.dtype], nb, BS, bt.data_ptr(), lib_mod.INDEX_I32, bt.stride(0), bt.shape[1],
            cl.data_ptr(), lib_mod.INDEX_I64, q.shape[0], H, KVH, D, 1.0 / math.sqrt(D),
            out.data_ptr(), out.stride(0), out.stride(1)]


def decode_with_workspace(lib, inputs, H, KVH, D, BS, splits):
    q, kc, vc, bt, cl = inputs
    out = torch.empty_like(q)
    n = lib.mkv_paged_decode_workspace_bytes(q.shape[0], H, KVH, D, BS, bt.shape[1], splits)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device="cuda")
    st = lib.mkv_paged_decode(*common_args(q, kc, vc, bt, cl, H, KVH, D, BS, out), ws.data_ptr(), n,
                              splits, None, torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.mkv_last_error()
    return out


def decode_no_alloc(lib, inputs, H, KVH, D, BS, splits):
    q, kc, vc, bt, cl = inputs
    out = torch.empty_like(q)
    st = lib.mkv_paged_decode_noalloc(*common_args(q, kc, vc, bt, cl, H, KVH, D, BS, out), splits,
                                      None, torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib.mkv_last_error()
    return out


@pytest.mark.parametrize("dtype,splits", [(torch.bfloat16, 0), (torch.bfloat16, 7), (torch.float32, 5)])
def test_no_alloc_matches_workspace_entry_twice(dtype, splits):
    lib = lib_mod.load()
    H, KVH, D, BS = 32, 8, 128, 16
    cases = [paged_inputs(24, H, KVH, D, BS, [1, 2000, 17, 640, 0, 1500] * 4, dtype, seed=1),
             paged_inputs(24, H, KVH, D, BS, [1999, 3, 300, 64, 1200, 511] * 4, dtype, seed=2)]
    for inputs in cases:  # two calls in a row: the second must not see the first's scratch
        q = inputs[0]
        need = lib.mkv_paged_decode_workspace_bytes(q.shape[0], H, KVH, D, BS, inputs[3].shape[1], splits)
        assert 0 < need <= lib_mod.NOALLOC_SCRATCH_BYTES  # the scratch is really used
        got = decode_no_alloc(lib, inputs, H, KVH, D, BS, splits)
        ref = decode_with_workspace(lib, inputs, H, KVH, D, BS, splits)
        torch.cuda.synchronize()
        atol, rtol = TOL[dtype]
        assert torch.equal(torch.isnan(got), torch.isnan(ref))
        ok = ~torch.isnan(ref)
        assert torch.allclose(got[ok].float(), ref[ok].float(), atol=atol, rtol=rtol)


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    lib = lib_mod.load()
    # config-3 sized batch with 8 fixed splits per sequence needs ~34 MB > 16 MiB
    need = lib.mkv_paged_decode_workspace_bytes(256, 32, 8, 128, 256, 32, 8)
    assert need > lib_mod.NOALLOC_SCRATCH_BYTES
    dummy = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    p = dummy.data_ptr()
    st = lib.mkv_paged_decode_noalloc(p, 4096, 128, lib_mod.DTYPE_BF16, p, p, lib_mod.DTYPE_BF16, 1,
                                      256, p, lib_mod.INDEX_I32, 32, 32, p, lib_mod.INDEX_I64, 256, 32,
                                      8, 128, 0.1, p, 4096, 128, 8, None,
                                      torch.cuda.current_stream().cuda_stream)
    assert st == lib_mod.ERR_WORKSPACE
    assert b"built-in scratch" in lib.mkv_last_error()
