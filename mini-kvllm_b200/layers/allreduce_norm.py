"""Tensor-parallel all-reduce fused with the residual add and RMSNorm that follow it.

In the reference, the row-parallel projections (o_proj, down_proj) end with
`dist.all_reduce(result)` (src/myvllm/layers/linear.py:222-225). The next LayerNorm call
then computes `s = x + residual; out = s / sqrt(mean(s^2) + eps) * weight` and returns
`(out, s)` (src/myvllm/layers/layernorm.py:17-27). `AllReduceResidualRMSNorm` does both
in one kernel (`mkv_allreduce_residual_rmsnorm`) over NVLink peer memory:
- The kernel copies each rank's partial product into one of two exchange buffers that
  the other ranks have mapped with CUDA IPC.
- Every rank reads all partials with peer loads, sums them in fp32 in rank order
  (identical bits everywhere), adds the residual and normalises.

Usage per step, on every rank in the same order:

    buf = ar.next_partial(num_tokens)          # a partial buffer at a fixed address
    torch.matmul(x, w_shard.t(), out=buf)      # (any tensor of that shape works too)
    out, residual = ar(buf, residual, weight)  # residual is updated in place

The call count lives on the device, so the sequence can be captured in a CUDA graph.

Partials larger than `oneshot_bytes` are summed with NCCL, and the kernel then runs as
residual add + RMSNorm only. Sizes beyond the buffers follow the same route. A rank
that stops answering makes the others' kernels time out (`timeout_ms`) instead of
hanging: they set an error flag, which `check()` turns into an exception.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from .. import _lib

_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}
_CYCLES_PER_MS = 2_000_000  # SM clock at most ~2 GHz: a bound, not a measurement


class AllReduceResidualRMSNorm:
    """Fused TP all-reduce + residual add + RMSNorm for one process group.

    max_tokens x hidden bounds the one-shot path. The two exchange buffers, the
    handshake flags and the call counter live in one IPC allocation per rank.
    Construction is collective: every rank of `group` must construct the object."""

    def __init__(self, max_tokens: int, hidden: int, dtype: torch.dtype = torch.bfloat16,
                 group=None, device: torch.device | None = None, timeout_ms: float = 1000.0,
                 oneshot_bytes: int = 4 << 20):
        if dtype not in _DTYPES:
            raise ValueError(f"AllReduceResidualRMSNorm: dtype must be bf16 or f16 (got {dtype})")
        if hidden % 8 != 0:
            raise ValueError(f"AllReduceResidualRMSNorm: hidden must be a multiple of 8 (got {hidden})")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if self.world > _lib.AR_MAX_RANKS:
            raise ValueError(f"AllReduceResidualRMSNorm: at most {_lib.AR_MAX_RANKS} ranks")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.max_tokens, self.hidden, self.dtype = max_tokens, hidden, dtype
        self.oneshot_bytes = oneshot_bytes
        self.timeout_cycles = int(timeout_ms * _CYCLES_PER_MS)
        self.error = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._solo_state = torch.zeros(2, dtype=torch.int32, device=self.device)  # world-1 calls
        self._lib = _lib.load()
        esz = self._esz = torch.tensor([], dtype=dtype).element_size()
        self._data_bytes = (max_tokens * hidden * esz + 255) // 256 * 256
        total = 2 * self._data_bytes + _lib.AR_FLAG_BYTES + 256  # 2 exchange buffers | flags | counter
        self._staging = torch.empty(max_tokens, hidden, dtype=dtype, device=self.device)
        self._own = ctypes.c_void_p()
        self._opened: list[int] = []
        if self.world == 1:
            return
        handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        with torch.cuda.device(self.device):
            _lib.check("mkv_ipc_alloc", self._lib.mkv_ipc_alloc(total, ctypes.byref(self._own), handle))
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            self.base = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.base.append(self._own.value)
                    continue
                ptr = ctypes.c_void_p()
                hb = ctypes.create_string_buffer(h, _lib.IPC_HANDLE_BYTES)
                _lib.check("mkv_ipc_open", self._lib.mkv_ipc_open(hb, ctypes.byref(ptr)))
                self._opened.append(ptr.value)
                self.base.append(ptr.value)
        self._peers = (ctypes.c_void_p * _lib.AR_MAX_RANKS)(*self.base)
        self._flags = (ctypes.c_void_p * _lib.AR_MAX_RANKS)(*[b + 2 * self._data_bytes for b in self.base])
        self._state = self.base[self.rank] + 2 * self._data_bytes + _lib.AR_FLAG_BYTES

    # ---------------------------------------------------------------- per call
    def _oneshot(self, num_tokens: int) -> bool:
        return (self.world > 1 and num_tokens <= self.max_tokens and
                num_tokens * self.hidden * self._esz <= self.oneshot_bytes)

    def next_partial(self, num_tokens: int) -> torch.Tensor:
        """A buffer for this rank's next partial, (num_tokens, hidden), at the same
        address every call up to max_tokens (any contiguous tensor may be passed instead)."""
        if num_tokens > self.max_tokens:
            return torch.empty(num_tokens, self.hidden, dtype=self.dtype, device=self.device)
        return self._staging[:num_tokens]

    def __call__(self, partial: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor,
                 eps: float = 1e-6) -> tuple[torch.Tensor, torch.Tensor]:
        """out = RMSNorm(all_reduce(partial) + residual) * weight; residual <- the sum
        (in place), as LayerNorm.residual_rms_forward returns it. Returns (out, sum).
        Without a residual the all-reduced partial itself is normalised, and the sum is
        a new tensor."""
        T, H = partial.shape
        if H != self.hidden or partial.dtype != self.dtype:
            raise ValueError("AllReduceResidualRMSNorm: partial must be (num_tokens, hidden) in the set dtype")
        for name, t in (("residual", residual), ("weight", weight)):
            if t is not None and (t.dtype != self.dtype or not t.is_contiguous()):
                raise ValueError(f"AllReduceResidualRMSNorm: {name} must be contiguous {self.dtype}")
        out = torch.empty_like(partial)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        partial = partial.contiguous()
        if self._oneshot(T):
            peers, flags, world, rank, state = self._peers, self._flags, self.world, self.rank, self._state
        else:
            if self.world > 1:
                dist.all_reduce(partial, group=self.group)
            peers, flags, world, rank, state = None, None, 1, 0, self._solo_state.data_ptr()
        res_out = residual if residual is not None else torch.empty_like(out)
        st = self._lib.mkv_allreduce_residual_rmsnorm(
            partial.data_ptr(), peers, self._data_bytes, flags, rank, world, state,
            residual.data_ptr() if residual is not None else None,
            res_out.data_ptr(), weight.data_ptr(), out.data_ptr(), T, H, _DTYPES[self.dtype],
            float(eps), self.error.data_ptr(), self.timeout_cycles, stream)
        _lib.check("mkv_allreduce_residual_rmsnorm", st)
        return out, res_out

    def check(self) -> None:
        """Raises if a handshake timed out since the last check (synchronises)."""
        if int(self.error.item()) != 0:
            self.error.zero_()
            raise RuntimeError("AllReduceResidualRMSNorm: a peer did not answer within the timeout")

    def close(self) -> None:
        for ptr in self._opened:
            self._lib.mkv_ipc_close(ctypes.c_void_p(ptr))
        self._opened = []
        if self._own.value:
            self._lib.mkv_ipc_free(self._own)
            self._own = ctypes.c_void_p()
