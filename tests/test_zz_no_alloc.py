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


def test_no_alloc_in_a_second_context():
    """A caller with its own driver-API context (a cgo/JNI host that created the context
    itself) gets the scratch address of that context, not the one cached for the
    primary context, and the primary context's calls stay correct afterwards."""
    drv = pytest.importorskip("cuda.bindings.driver")

    def ok(res):
        res = res if isinstance(res, tuple) else (res,)
        assert res[0] == drv.CUresult.CUDA_SUCCESS, res[0]
        return res[1] if len(res) == 2 else res[1:]

    lib = lib_mod.load()
    H, KVH, D, BS, splits = 32, 8, 128, 16, 7
    inputs = paged_inputs(24, H, KVH, D, BS, [1, 2000, 17, 640, 0, 1500] * 4, torch.bfloat16, seed=3)
    q, kc, vc, bt, cl = inputs
    ref = decode_with_workspace(lib, inputs, H, KVH, D, BS, splits)
    first = decode_no_alloc(lib, inputs, H, KVH, D, BS, splits)  # caches the primary's address
    torch.cuda.synchronize()
    host = [t.view(torch.uint8).cpu().numpy() if t.dtype != torch.bfloat16 else
            t.view(torch.int16).cpu().numpy() for t in (q, kc, vc, bt, cl)]

    ok(drv.cuInit(0))
    dev = ok(drv.cuDeviceGet(torch.cuda.current_device()))
    ctx = ok(drv.cuCtxCreate(0, dev))  # now current on this thread
    ptrs = []
    try:
        for h in host:
            p = ok(drv.cuMemAlloc(h.nbytes))
            ok(drv.cuMemcpyHtoD(p, h.ctypes.data, h.nbytes))
            ptrs.append(p)
        out_bytes = q.numel() * 2
        optr = ok(drv.cuMemAlloc(out_bytes))
        ptrs.append(optr)
        dq, dk, dv, dbt, dcl = (int(p) for p in ptrs[:5])
        results = []
        for _ in range(2):  # two calls in a row in this context
            st = lib.mkv_paged_decode_noalloc(
                dq, q.stride(0), q.stride(1), lib_mod.DTYPE_BF16, dk, dv, lib_mod.DTYPE_BF16,
                kc.shape[0], BS, dbt, lib_mod.INDEX_I32, bt.stride(0), bt.shape[1], dcl,
                lib_mod.INDEX_I64, q.shape[0], H, KVH, D, 1.0 / math.sqrt(D), int(optr), q.stride(0),
                q.stride(1), splits, None, None)
            assert st == 0, lib.mkv_last_error()
            ok(drv.cuCtxSynchronize())
            buf = torch.empty(q.shape, dtype=torch.bfloat16)
            ok(drv.cuMemcpyDtoH(buf.data_ptr(), optr, out_bytes))
            results.append(buf)
    finally:
        for p in ptrs:
            drv.cuMemFree(p)
        drv.cuCtxDestroy(ctx)
    torch.cuda.set_device(torch.cuda.current_device())
    again = decode_no_alloc(lib, inputs, H, KVH, D, BS, splits)  # primary context again
    torch.cuda.synchronize()
    atol, rtol = TOL[torch.bfloat16]
    ok_rows = ~torch.isnan(ref.cpu())
    for got in results + [first.cpu(), again.cpu()]:
        assert torch.equal(torch.isnan(got), ~ok_rows)
        assert torch.allclose(got[ok_rows].float(), ref.cpu()[ok_rows].float(), atol=atol, rtol=rtol)
