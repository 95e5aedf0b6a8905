"""The fused tensor-parallel all-reduce + residual add + RMSNorm
(`mkv_allreduce_residual_rmsnorm`, `layers/allreduce_norm.py`) against the oracle
`allreduce_residual_rmsnorm_ref`, which is pinned to the reference's
LayerNorm.residual_rms_forward by tests/golden/residual_rmsnorm.npz.

- World size 1: residual add + RMSNorm of one partial.
- N ranks emulated on one GPU: N partial buffers and flag arrays on the same device,
  with every rank's flags already set. Each emulated rank is one launch that waits for
  nothing, so no kernel depends on another launch. The outputs must be bit-identical
  across ranks.
- Timeout: a flag that nothing sets makes the handshake give up, set the error flag,
  and leave the context usable.
- Real ranks: with two or more GPUs, two processes under torchrun check against NCCL
  and the oracle (`mini-kvllm_b200/bench_allreduce_norm.py --check`).

Tolerance: the sum and the residual output bit-exact; the normalised output within
atol 2e-2 / rtol 1e-2 (bf16)."""
import ctypes
import os
import subprocess
import sys

import pytest
import torch

from conftest import REPO, mkv_module
from oracle import allreduce_residual_rmsnorm_ref

pytestmark = pytest.mark.gpu
lib_mod = mkv_module("_lib")
arn = mkv_module("layers.allreduce_norm")


def _close(out, ref):
    assert torch.allclose(out.float().cpu(), ref.float(), atol=2e-2, rtol=1e-2), \
        f"max abs err {float((out.float().cpu() - ref.float()).abs().max()):.3e}"


@pytest.mark.parametrize("T,H", [(1, 1024), (37, 1024), (256, 4096), (300, 8192), (5, 8)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_residual", [True, False])
def test_world1_matches_oracle(T, H, dtype, with_residual):
    g = torch.Generator().manual_seed(T + H)
    x = torch.randn(1, T, H, generator=g).to(dtype)
    res = (torch.randn(T, H, generator=g) * 2).to(dtype) if with_residual else None
    w = (torch.rand(H, generator=g) + 0.5).to(dtype)
    ar = arn.AllReduceResidualRMSNorm(T, H, dtype=dtype)
    r_dev = res.cuda() if res is not None else None
    out, s = ar(x[0].cuda(), r_dev, w.cuda(), eps=1e-6)
    torch.cuda.synchronize()
    ref_out, ref_s = allreduce_residual_rmsnorm_ref(x, res, w, 1e-6, dtype)
    assert torch.equal(s.cpu(), ref_s)
    if with_residual:
        assert s.data_ptr() == r_dev.data_ptr()  # updated in place
    _close(out, ref_out)


def _emulated_call(lib, partials, xbufs, flags, rank, state, residual, weight, out, err, timeout_cycles=0):
    """Rank `rank` of len(partials) emulated ranks: xbufs[r] holds rank r's two exchange
    buffers (2, T, H), flags[r] its flag array."""
    N = len(partials)
    peers = (ctypes.c_void_p * 8)(*[x.data_ptr() for x in xbufs])
    fl = (ctypes.c_void_p * 8)(*[f.data_ptr() for f in flags])
    T, H = partials[0].shape
    code = lib_mod.DTYPE_BF16 if partials[0].dtype == torch.bfloat16 else lib_mod.DTYPE_F16
    st = lib.mkv_allreduce_residual_rmsnorm(
        partials[rank].data_ptr(), peers, xbufs[0][0].numel() * xbufs[0].element_size(), fl, rank, N,
        state.data_ptr(), residual.data_ptr() if residual is not None else None,
        residual.data_ptr() if residual is not None else None, weight.data_ptr(), out.data_ptr(),
        T, H, code, 1e-6, err.data_ptr(), timeout_cycles,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.mkv_last_error()


@pytest.mark.parametrize("N", [2, 4, 8])
@pytest.mark.parametrize("T", [1, 64, 200])
def test_emulated_ranks_match_oracle_and_each_other(N, T):
    lib = lib_mod.load()
    H, dtype = 1024, torch.bfloat16
    g = torch.Generator().manual_seed(N * 1000 + T)
    parts = torch.randn(N, T, H, generator=g).to(dtype)
    res = (torch.randn(T, H, generator=g) * 2).to(dtype)
    w = (torch.rand(H, generator=g) + 0.5).to(dtype)
    partials = [parts[r].cuda().contiguous() for r in range(N)]
    epoch = 7  # odd: exchange buffer 1
    # each emulated rank's exchange buffers already hold its partial (as its own call would
    # have copied it); the kernel copies this rank's again
    # every rank's arrive and depart flags already hold this call's epoch from every source;
    # each emulated rank keeps its call counter at epoch - 1
    flags = [torch.full((lib_mod.AR_FLAG_BYTES // 4,), epoch, dtype=torch.int32, device="cuda") for _ in range(N)]
    states = [torch.tensor([epoch - 1, 0], dtype=torch.int32, device="cuda") for _ in range(N)]
    xbufs = [torch.zeros(2, T, H, dtype=dtype, device="cuda") for _ in range(N)]
    for r in range(N):
        xbufs[r][epoch & 1].copy_(partials[r])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref_out, ref_s = allreduce_residual_rmsnorm_ref(parts, res, w, 1e-6, dtype)
    outs = []
    for r in range(N):
        residual = res.cuda()
        out = torch.empty(T, H, dtype=dtype, device="cuda")
        _emulated_call(lib, partials, xbufs, flags, r, states[r], residual, w.cuda(), out, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert states[r].tolist() == [epoch, 0]  # the call counter advanced, the block count reset
        assert torch.equal(residual.cpu(), ref_s)
        _close(out, ref_out)
        outs.append(out)
    for r in range(1, N):
        assert torch.equal(outs[r], outs[0])  # every rank computes the same bits


def test_handshake_timeout_sets_error_flag():
    """A peer that never signals: the wait gives up after ~1e6 cycles, sets the error
    flag, and the next call on the same context works."""
    lib = lib_mod.load()
    T, H = 4, 1024
    partials = [torch.randn(T, H, device="cuda").bfloat16() for _ in range(2)]
    flags = [torch.zeros(lib_mod.AR_FLAG_BYTES // 4, dtype=torch.int32, device="cuda") for _ in range(2)]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    w = torch.ones(H, device="cuda").bfloat16()
    out = torch.empty(T, H, device="cuda").bfloat16()
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    xbufs = [torch.zeros(2, T, H, device="cuda").bfloat16() for _ in range(2)]
    _emulated_call(lib, partials, xbufs, flags, 0, state, None, w, out, err, timeout_cycles=1_000_000)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    # the context is still usable: world size 1 on the same buffers
    ar = arn.AllReduceResidualRMSNorm(T, H)
    o, _ = ar(partials[0], None, w)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_over_nvlink(tmp_path):
    """Two processes, one GPU each: every rank's sum bit-exact against the oracle over all
    ranks' partials, the output within tolerance, and all ranks bit-identical."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    tokens = "1,37,256,2048"  # 2048 x 1024 bf16 = 4 MiB: still one-shot
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29631",
           os.path.join(REPO, "mini-kvllm_b200", "bench_allreduce_norm.py"), "--check",
           "--dump", str(tmp_path), "--tokens", tokens, "--iters", "20"]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "check ok" in r.stdout
    for T in [int(t) for t in tokens.split(",")]:
        d = [torch.load(tmp_path / f"rank{k}_T{T}.pt") for k in range(2)]
        parts = torch.stack([x["partial"] for x in d])
        ref_out, ref_s = allreduce_residual_rmsnorm_ref(parts, d[0]["residual"], d[0]["weight"], d[0]["eps"])
        for x in d:
            assert torch.equal(x["sum"], ref_s)
            _close(x["out"], ref_out)
