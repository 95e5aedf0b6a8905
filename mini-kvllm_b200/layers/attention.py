"""Drop-in replacements for mini-kvllm's paged KV-cache hot path.

The functions keep the reference's names, argument order and meaning
(heart1128/mini-kvllm, src/myvllm/layers/attention.py):

  store_kvcache(key, value, k_cache, v_cache, slot_mapping, block_size)           # :67
  store_kvcache_int8(key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping,
                     block_size)                                                   # :255
  store_kvcache_fp8(key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping,
                    block_size, kv_cache_dtype)                                    # :281
  paged_attention_decode(query, k_cache, v_cache, block_tables, context_lens, scale,
                         num_heads, num_kv_heads, head_dim, block_size)            # :895
  paged_attention_decode_quantized(query, k_cache, v_cache, k_scale, v_scale,
                         block_tables, context_lens, scale, num_heads, num_kv_heads,
                         head_dim, block_size, kv_cache_dtype)                     # :1213
  paged_attention_prefill(query, k_cache, v_cache, block_tables, context_lens,
                          cu_seqlens_q, positions, scale, num_heads, num_kv_heads,
                          head_dim, block_size)        # paged_attention_prefill_triton :852

with kv_cache_dtype "fp8_per_tensor" (scales of shape (1,)), "fp8_per_token_head" and
"int8_per_token_head" (scales of shape (num_blocks, block_size, num_kv_heads)).

and `Attention` keeps the module contract of attention.py:1617-1807 (cache tensors and
scales injected as attributes by the model runner, metadata read from the global
context). Each call maps tensors to raw pointers and strides and launches the sm_100a
kernels of libmkv.so on the current CUDA stream; there is no Triton, no CPU path and
no fallback. Nothing synchronises with the host, so the decode step (append + decode)
can be captured in a CUDA graph, including the FP8 path whose per-tensor scale is
calibrated on the device.
"""
from __future__ import annotations

import ctypes
import os

import torch
from torch import nn

from .. import _lib
from ..utils.context import get_context

FP8_E4M3_MAX = 448.0

_DTYPES = {
    torch.float32: _lib.DTYPE_F32,
    torch.float16: _lib.DTYPE_F16,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float8_e4m3fn: _lib.DTYPE_FP8_E4M3,
    torch.int8: _lib.DTYPE_INT8,
}
_PER_TOKEN_HEAD = ("fp8_per_token_head", "int8_per_token_head")
_INDEX = {torch.int32: _lib.INDEX_I32, torch.int64: _lib.INDEX_I64}
_FLOAT_IO = (torch.float32, torch.float16, torch.bfloat16)


class _on_device:
    """Makes `device` current for the duration of a launch (no-op when it already is)."""

    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def _require_cuda(fn: str, *tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise ValueError(f"{fn}: all tensors must be CUDA tensors (got {t.device})")
        if t.device != dev:
            raise ValueError(f"{fn}: tensors are on different devices ({dev} and {t.device})")
    return dev


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _index_tensor(t: torch.Tensor, fn: str, what: str) -> torch.Tensor:
    if t.dtype not in _INDEX:
        raise ValueError(f"{fn}: {what} must be int32 or int64 (got {t.dtype})")
    return t if t.is_contiguous() else t.contiguous()


def _row_major_tokens(x: torch.Tensor) -> torch.Tensor:
    """(T, KVH, D) view whose last dim is contiguous (strides of dims 0/1 may be anything)."""
    return x if x.stride(-1) == 1 else x.contiguous()


def _check_cache(fn: str, k_cache: torch.Tensor, v_cache: torch.Tensor, block_size: int,
                 num_kv_heads: int, head_dim: int) -> int:
    if k_cache.shape != v_cache.shape or k_cache.dtype != v_cache.dtype:
        raise ValueError(f"{fn}: K and V cache shapes/dtypes must match")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError(f"{fn}: caches must be contiguous (num_blocks, block_size, num_kv_heads, head_dim)")
    row = block_size * num_kv_heads * head_dim
    if row <= 0 or k_cache.numel() % row != 0:
        raise ValueError(f"{fn}: cache of shape {tuple(k_cache.shape)} is not a whole number of "
                         f"({block_size}, {num_kv_heads}, {head_dim}) blocks")
    return k_cache.numel() // row


# ---------------------------------------------------------------------------------- append
def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor, block_size: int) -> None:
    """Stores key/value (num_tokens, num_kv_heads, head_dim) into the paged caches
    (num_blocks, block_size, num_kv_heads, head_dim) at slot_mapping[t]; slot -1 skips
    the token. Reference: attention.py:67-108 (kernel 7-64)."""
    fn = "store_kvcache"
    num_tokens, num_kv_heads, head_dim = key.shape
    assert k_cache.shape == v_cache.shape, "K and V cache shapes must match"
    assert slot_mapping.numel() == num_tokens, "Slot mapping size must match number of tokens"
    dev = _require_cuda(fn, key, value, k_cache, v_cache, slot_mapping)
    if k_cache.dtype not in _DTYPES:
        raise ValueError(f"{fn}: unsupported cache dtype {k_cache.dtype}")
    key, value = _row_major_tokens(key), _row_major_tokens(value)
    if key.dtype != k_cache.dtype:  # the reference's tl.store converts to the cache dtype
        key, value = key.to(k_cache.dtype), value.to(k_cache.dtype)
    num_blocks = _check_cache(fn, k_cache, v_cache, block_size, num_kv_heads, head_dim)
    slots = _index_tensor(slot_mapping.reshape(-1), fn, "slot_mapping")
    lib = _lib.load()
    with _on_device(dev):
        st = lib.mkv_store_kvcache(
            key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1),
            value.stride(0), value.stride(1), k_cache.data_ptr(), v_cache.data_ptr(),
            num_blocks, block_size, slots.data_ptr(), _INDEX[slots.dtype], num_tokens,
            num_kv_heads, head_dim, _DTYPES[k_cache.dtype], None, _stream(dev))
    _lib.check(fn, st)


_calib_work: dict[int, torch.Tensor] = {}


_calibration_suspended = 0


class fp8_calibration_suspended:
    """Context manager: FP8 appends inside it quantise with the scales as they are and do
    not calibrate a scale that still holds the 1.0 sentinel.

    For a model runner's eager warm-up before CUDA-graph capture. The reference runner
    (model_runner.py:783-795) calls the model once on dummy decode inputs before
    capturing, which would otherwise calibrate the per-tensor scale from dummy K/V and
    freeze it. The capture itself records the calibration kernel as usual, so the first
    replay on real data still calibrates. Nests; not tied to a thread or stream."""

    def __enter__(self):
        global _calibration_suspended
        _calibration_suspended += 1
        return self

    def __exit__(self, *exc):
        global _calibration_suspended
        _calibration_suspended -= 1
        return False


def _calibration_work(device: torch.device) -> torch.Tensor:
    """Per-device 16-byte scratch of the FP8 calibration kernel (zero between calls)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _calib_work.get(idx)
    if buf is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                "store_kvcache_fp8: run one FP8 append eagerly on this device before CUDA-graph "
                "capture (its calibration scratch must be allocated outside the capture)")
        buf = torch.zeros(_lib.FP8_CALIB_WORK_BYTES, dtype=torch.uint8, device=device)
        _calib_work[idx] = buf
    return buf


def store_kvcache_fp8(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                      v_cache: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
                      slot_mapping: torch.Tensor, block_size: int, kv_cache_dtype: str) -> None:
    """Quantises key/value to FP8 E4M3 with per-tensor scales and stores them into the
    paged caches. While a scale still holds the sentinel 1.0 it is first calibrated from
    this batch (bf16/fp16/fp32 amax / 448, computed on the device); afterwards it stays
    frozen. Reference: attention.py:281-333 (calibration 315-323, kernel 118-191)."""
    fn = "store_kvcache_fp8"
    if kv_cache_dtype == "fp8_per_token_head":
        return _store_per_token_head(fn, key, value, k_cache, v_cache, k_scale, v_scale,
                                     slot_mapping, block_size, _lib.DTYPE_FP8_E4M3)
    if kv_cache_dtype != "fp8_per_tensor":
        raise NotImplementedError(
            f"{fn}: kv_cache_dtype {kv_cache_dtype!r} is not implemented "
            "('fp8_per_tensor' or 'fp8_per_token_head')")
    num_tokens, num_kv_heads, head_dim = key.shape
    dev = _require_cuda(fn, key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping)
    if key.dtype not in _FLOAT_IO or value.dtype != key.dtype:
        raise ValueError(f"{fn}: key/value must share a float32/float16/bfloat16 dtype")
    if k_cache.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise ValueError(f"{fn}: caches must be float8_e4m3fn (got {k_cache.dtype})")
    if k_scale.dtype != torch.float32 or v_scale.dtype != torch.float32 or \
            k_scale.numel() < 1 or v_scale.numel() < 1:
        raise ValueError(f"{fn}: k_scale/v_scale must be float32 tensors with one element")
    assert slot_mapping.numel() == num_tokens, "Slot mapping size must match number of tokens"
    key, value = _row_major_tokens(key), _row_major_tokens(value)
    num_blocks = _check_cache(fn, k_cache, v_cache, block_size, num_kv_heads, head_dim)
    slots = _index_tensor(slot_mapping.reshape(-1), fn, "slot_mapping")
    lib = _lib.load()
    dt = _DTYPES[key.dtype]
    with _on_device(dev):
        # one launch: calibration of a sentinel scale (unless suspended) + quantising store
        work = None if _calibration_suspended else _calibration_work(dev).data_ptr()
        st = lib.mkv_store_kvcache_fp8_calibrating(
            key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1), value.stride(0),
            value.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), k_scale.data_ptr(),
            v_scale.data_ptr(), num_blocks, block_size, slots.data_ptr(), _INDEX[slots.dtype],
            num_tokens, num_kv_heads, head_dim, dt, work, None, _stream(dev))
    _lib.check(fn, st)


def _check_row_scales(fn: str, k_scale: torch.Tensor, v_scale: torch.Tensor, num_blocks: int,
                      block_size: int, num_kv_heads: int) -> None:
    n = num_blocks * block_size * num_kv_heads
    for name, t in (("k_scale", k_scale), ("v_scale", v_scale)):
        if t.dtype != torch.float32 or t.numel() != n or not t.is_contiguous():
            raise ValueError(f"{fn}: {name} must be a contiguous float32 tensor of "
                             f"(num_blocks, block_size, num_kv_heads) = {n} elements")


def _store_per_token_head(fn, key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping,
                          block_size, cache_code):
    num_tokens, num_kv_heads, head_dim = key.shape
    dev = _require_cuda(fn, key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping)
    if key.dtype not in _FLOAT_IO or value.dtype != key.dtype:
        raise ValueError(f"{fn}: key/value must share a float32/float16/bfloat16 dtype")
    want = torch.int8 if cache_code == _lib.DTYPE_INT8 else (torch.float8_e4m3fn, torch.uint8)
    if (k_cache.dtype != want) if isinstance(want, torch.dtype) else (k_cache.dtype not in want):
        raise ValueError(f"{fn}: caches have dtype {k_cache.dtype}, expected {want}")
    assert slot_mapping.numel() == num_tokens, "Slot mapping size must match number of tokens"
    key, value = _row_major_tokens(key), _row_major_tokens(value)
    num_blocks = _check_cache(fn, k_cache, v_cache, block_size, num_kv_heads, head_dim)
    _check_row_scales(fn, k_scale, v_scale, num_blocks, block_size, num_kv_heads)
    slots = _index_tensor(slot_mapping.reshape(-1), fn, "slot_mapping")
    lib = _lib.load()
    with _on_device(dev):
        st = lib.mkv_store_kvcache_quant_per_token_head(
            key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1), value.stride(0),
            value.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), cache_code,
            k_scale.data_ptr(), v_scale.data_ptr(), num_blocks, block_size, slots.data_ptr(),
            _INDEX[slots.dtype], num_tokens, num_kv_heads, head_dim, _DTYPES[key.dtype], None,
            _stream(dev))
    _lib.check(fn, st)


def store_kvcache_int8(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                       v_cache: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
                       slot_mapping: torch.Tensor, block_size: int) -> None:
    """Quantises each (token, kv head) row of key/value to INT8 with its own scale
    max(amax / 127, 1e-6) (x * (1 / scale), rounded half away from zero, clamped to
    [-128, 127]) and stores it into the int8 paged caches, writing the scale into
    k_scale/v_scale (num_blocks, block_size, num_kv_heads) at the token's slot.
    Reference: attention.py:255-278 (kernel 195-252)."""
    _store_per_token_head("store_kvcache_int8", key, value, k_cache, v_cache, k_scale, v_scale,
                          slot_mapping, block_size, _lib.DTYPE_INT8)


# ---------------------------------------------------------------------------------- decode
_decode_ws: dict[tuple[int, int], torch.Tensor] = {}
_decode_ctr: dict[tuple[int, int], torch.Tensor] = {}


def _decode_buffers(dev: torch.device, stream_ptr: int, ws_bytes: int, ctr_bytes: int):
    """(workspace, counters) for a decode on `stream_ptr`, kept per (device, stream).
    The counter buffer holds nothing but the split merge's arrival counters: it is zeroed
    when allocated and every decode leaves it zero, so decodes ordered on that stream
    share it with no clearing. The workspace holds the partials (no initial value). Inside
    a CUDA-graph capture a buffer too small is not replaced: the call takes a fresh
    workspace from the capture's pool and passes no counter buffer, so the library clears
    the counters in the graph."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (idx, stream_ptr)
    ws, ctr = _decode_ws.get(key), _decode_ctr.get(key)
    ws_ok = ws is not None and ws.numel() >= ws_bytes
    ctr_ok = ctr is not None and ctr.numel() >= ctr_bytes
    if (ws_ok and ctr_ok) or ws_bytes == 0:
        return (ws if ws_bytes else None), (ctr if ctr_bytes else None)
    if torch.cuda.is_current_stream_capturing():
        return torch.empty(ws_bytes, dtype=torch.uint8, device=dev), None
    if not ws_ok:
        ws = torch.empty(max(ws_bytes, 1 << 20), dtype=torch.uint8, device=dev)
        _decode_ws[key] = ws
    if not ctr_ok:
        ctr = torch.zeros(max(ctr_bytes, 64 << 10), dtype=torch.uint8, device=dev)
        _decode_ctr[key] = ctr
    return ws, ctr


def _decode(fn: str, query, k_cache, v_cache, k_scale, v_scale, block_tables, context_lens,
            scale, num_heads, num_kv_heads, head_dim, block_size, num_splits: int = 0,
            per_token_head: bool = False, overlap_previous: bool = False):
    if query.dim() != 3 or query.shape[1] != num_heads or query.shape[2] != head_dim:
        raise ValueError(f"{fn}: query must be (batch, {num_heads}, {head_dim}), got {tuple(query.shape)}")
    if query.dtype not in _FLOAT_IO:
        raise ValueError(f"{fn}: unsupported query dtype {query.dtype}")
    tensors = [query, k_cache, v_cache, block_tables, context_lens]
    if k_scale is not None:
        tensors += [k_scale, v_scale]
    dev = _require_cuda(fn, *tensors)
    batch_size = query.shape[0]
    max_num_blocks = block_tables.shape[1]
    inputs = (query.data_ptr(), block_tables.data_ptr(), context_lens.data_ptr())
    query = query if query.stride(-1) == 1 else query.contiguous()
    output = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    if batch_size == 0:
        return output
    if block_tables.stride(-1) != 1:
        block_tables = block_tables.contiguous()
    if block_tables.dtype not in _INDEX:
        raise ValueError(f"{fn}: block_tables must be int32 or int64 (got {block_tables.dtype})")
    lens = _index_tensor(context_lens.reshape(-1), fn, "context_lens")
    if lens.numel() != batch_size or block_tables.shape[0] < batch_size:
        raise ValueError(f"{fn}: context_lens/block_tables do not cover {batch_size} sequences")
    num_blocks = _check_cache(fn, k_cache, v_cache, block_size, num_kv_heads, head_dim)
    if per_token_head:
        _check_row_scales(fn, k_scale, v_scale, num_blocks, block_size, num_kv_heads)
    # an input copied here was written by the kernel just launched: no overlap with it
    copied = inputs != (query.data_ptr(), block_tables.data_ptr(), lens.data_ptr())
    lib = _lib.load()
    ws_bytes = lib.mkv_paged_decode_workspace_bytes(batch_size, num_heads, num_kv_heads, head_dim,
                                                    block_size, max_num_blocks, num_splits)
    ctr_bytes = lib.mkv_paged_decode_counter_bytes(batch_size, num_heads, num_kv_heads, head_dim,
                                                   block_size, max_num_blocks, num_splits)
    with _on_device(dev):
        stream = _stream(dev)
        ws, ctr = _decode_buffers(dev, stream.value or 0, ws_bytes, ctr_bytes)
        flags = _lib.DECODE_OVERLAP_PREVIOUS if overlap_previous and not copied else 0
        pt = k_scale is not None and not per_token_head  # per-tensor FP8 scales
        st = lib.mkv_paged_decode_ex(
            query.data_ptr(), query.stride(0), query.stride(1), _DTYPES[query.dtype],
            k_cache.data_ptr(), v_cache.data_ptr(),
            _lib.DTYPE_FP8_E4M3 if k_cache.dtype == torch.uint8 else _DTYPES[k_cache.dtype],
            k_scale.data_ptr() if pt else None, v_scale.data_ptr() if pt else None,
            k_scale.data_ptr() if per_token_head else None,
            v_scale.data_ptr() if per_token_head else None,
            num_blocks, block_size, block_tables.data_ptr(), _INDEX[block_tables.dtype],
            block_tables.stride(0), max_num_blocks, lens.data_ptr(), _INDEX[lens.dtype],
            batch_size, num_heads, num_kv_heads, head_dim, float(scale), output.data_ptr(),
            output.stride(0), output.stride(1), ws.data_ptr() if ws is not None else None,
            ws.numel() if ws is not None else 0, ctr.data_ptr() if ctr is not None else None,
            ctr.numel() if ctr is not None else 0, num_splits, flags, None, stream)
    _lib.check(fn, st)
    return output


def paged_attention_decode(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float,
                           num_heads: int, num_kv_heads: int, head_dim: int,
                           block_size: int, num_splits: int = 0,
                           overlap_previous: bool = False) -> torch.Tensor:
    """Decode attention of query (batch, num_heads, head_dim) over the paged K/V of each
    sequence: tokens t < context_lens[b] on pages block_tables[b, t // block_size],
    GQA kv head = h // (num_heads // num_kv_heads). Returns (batch, num_heads, head_dim)
    in the query dtype. Reference: attention.py:895-950 (kernel 517-646).
    `num_splits` (0 = automatic) forces the split-KV count; it is not in the reference.
    `overlap_previous` (not in the reference) lets the decode start while the previous
    kernel on the stream runs, reading the pages only once it has completed; pass it only
    when that kernel writes none of query, block_tables and context_lens, as when it is
    this step's store_kvcache (Attention.forward does so)."""
    if k_cache.dtype == torch.float8_e4m3fn:
        raise ValueError("paged_attention_decode: FP8 caches go through paged_attention_decode_quantized")
    return _decode("paged_attention_decode", query, k_cache, v_cache, None, None, block_tables,
                   context_lens, scale, num_heads, num_kv_heads, head_dim, block_size, num_splits,
                   overlap_previous=overlap_previous)


def paged_attention_decode_quantized(query: torch.Tensor, k_cache: torch.Tensor,
                                     v_cache: torch.Tensor, k_scale: torch.Tensor,
                                     v_scale: torch.Tensor, block_tables: torch.Tensor,
                                     context_lens: torch.Tensor, scale: float, num_heads: int,
                                     num_kv_heads: int, head_dim: int, block_size: int,
                                     kv_cache_dtype: str, num_splits: int = 0,
                                     overlap_previous: bool = False) -> torch.Tensor:
    """Decode attention over a quantised paged cache, dequantised while the pages are
    loaded: 'fp8_per_tensor' (e4m3 pages, scales of shape (1,)), 'fp8_per_token_head'
    (e4m3) and 'int8_per_token_head' (int8), the last two with a scale per (page, row,
    kv head) in k_scale/v_scale (num_blocks, block_size, num_kv_heads). Reference:
    attention.py:1213-1268 with paged_attention_decode_fp8_kernel (953-1121) and
    paged_attention_decode_quantized_tile_kernel (1124-1210). `num_splits` and
    `overlap_previous` as for paged_attention_decode."""
    fn = "paged_attention_decode_quantized"
    if kv_cache_dtype in _PER_TOKEN_HEAD:
        want = torch.int8 if kv_cache_dtype.startswith("int8") else torch.float8_e4m3fn
        if k_cache.dtype != want:
            raise ValueError(f"{fn}: {kv_cache_dtype} needs {want} caches (got {k_cache.dtype})")
        return _decode(fn, query, k_cache, v_cache, k_scale, v_scale, block_tables,
                       context_lens, scale, num_heads, num_kv_heads, head_dim, block_size,
                       num_splits, per_token_head=True, overlap_previous=overlap_previous)
    if kv_cache_dtype != "fp8_per_tensor":
        raise NotImplementedError(
            f"{fn}: kv_cache_dtype {kv_cache_dtype!r} is not implemented "
            "('fp8_per_tensor', 'fp8_per_token_head' or 'int8_per_token_head')")
    if k_cache.dtype not in (torch.float8_e4m3fn, torch.uint8):
        raise ValueError(f"{fn}: caches must be float8_e4m3fn (got {k_cache.dtype})")
    if k_scale.dtype != torch.float32 or v_scale.dtype != torch.float32:
        raise ValueError(f"{fn}: k_scale/v_scale must be float32")
    return _decode(fn, query, k_cache, v_cache, k_scale, v_scale, block_tables, context_lens,
                   scale, num_heads, num_kv_heads, head_dim, block_size, num_splits,
                   overlap_previous=overlap_previous)


# ---------------------------------------------------------------------------------- prefill
def paged_attention_prefill(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            block_tables: torch.Tensor, context_lens: torch.Tensor,
                            cu_seqlens_q: torch.Tensor, positions: torch.Tensor, scale: float,
                            num_heads: int, num_kv_heads: int, head_dim: int, block_size: int,
                            k_scale: torch.Tensor | None = None,
                            v_scale: torch.Tensor | None = None,
                            kv_cache_dtype: str = "auto") -> torch.Tensor:
    """Chunked-prefill / extend attention over the paged cache: query (total_q, num_heads,
    head_dim) holds every sequence's new tokens (sequence b owns rows
    [cu_seqlens_q[b], cu_seqlens_q[b+1])); row q at absolute position positions[q] sees the
    cached tokens t < min(context_lens[b], positions[q] + 1), so its own K/V must have
    been appended. Returns (total_q, num_heads, head_dim) in the query dtype. Reference:
    paged_attention_prefill_triton, attention.py:852-892 (kernel 704-849). The
    quantised caches ('fp8_per_tensor', 'fp8_per_token_head', 'int8_per_token_head'
    with their k_scale / v_scale) are extensions the reference lists as a TODO."""
    fn = "paged_attention_prefill"
    if query.dim() != 3 or query.shape[1] != num_heads or query.shape[2] != head_dim:
        raise ValueError(f"{fn}: query must be (total_q, {num_heads}, {head_dim}), got {tuple(query.shape)}")
    if query.dtype not in _FLOAT_IO:
        raise ValueError(f"{fn}: unsupported query dtype {query.dtype}")
    tensors = [query, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, positions]
    quant = kv_cache_dtype != "auto"
    if quant:
        if kv_cache_dtype not in ("fp8_per_tensor",) + _PER_TOKEN_HEAD:
            raise NotImplementedError(f"{fn}: kv_cache_dtype {kv_cache_dtype!r} is not implemented")
        if k_scale is None or v_scale is None:
            raise ValueError(f"{fn}: {kv_cache_dtype} needs k_scale and v_scale")
        tensors += [k_scale, v_scale]
    dev = _require_cuda(fn, *tensors)
    total_q = query.shape[0]
    query = query if query.stride(-1) == 1 and query.stride(1) % 8 == 0 and query.stride(0) % 8 == 0 \
        else query.contiguous()
    output = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    num_seqs = context_lens.numel()
    if total_q == 0 or num_seqs == 0:
        return output
    if block_tables.stride(-1) != 1:
        block_tables = block_tables.contiguous()
    if block_tables.dtype not in _INDEX:
        raise ValueError(f"{fn}: block_tables must be int32 or int64 (got {block_tables.dtype})")
    lens = _index_tensor(context_lens.reshape(-1), fn, "context_lens")
    cu = _index_tensor(cu_seqlens_q.reshape(-1), fn, "cu_seqlens_q")
    pos = _index_tensor(positions.reshape(-1), fn, "positions")
    if cu.numel() != num_seqs + 1 or pos.numel() != total_q or block_tables.shape[0] < num_seqs:
        raise ValueError(f"{fn}: cu_seqlens_q/positions/block_tables do not match "
                         f"{num_seqs} sequences and {total_q} query tokens")
    num_blocks = _check_cache(fn, k_cache, v_cache, block_size, num_kv_heads, head_dim)
    kp = vp = kps = vps = None
    if kv_cache_dtype == "fp8_per_tensor":
        if k_cache.dtype not in (torch.float8_e4m3fn, torch.uint8):
            raise ValueError(f"{fn}: fp8_per_tensor needs float8_e4m3fn caches (got {k_cache.dtype})")
        kp, vp = k_scale.data_ptr(), v_scale.data_ptr()
        cache_code = _lib.DTYPE_FP8_E4M3
    elif quant:
        want = torch.int8 if kv_cache_dtype.startswith("int8") else torch.float8_e4m3fn
        if k_cache.dtype != want:
            raise ValueError(f"{fn}: {kv_cache_dtype} needs {want} caches (got {k_cache.dtype})")
        _check_row_scales(fn, k_scale, v_scale, num_blocks, block_size, num_kv_heads)
        kps, vps = k_scale.data_ptr(), v_scale.data_ptr()
        cache_code = _DTYPES[want]
    else:
        if k_cache.dtype != query.dtype:
            raise ValueError(f"{fn}: cache dtype {k_cache.dtype} must equal the query dtype {query.dtype}")
        cache_code = _DTYPES[k_cache.dtype]
    lib = _lib.load()
    # 8-bit caches with long chunks: scratch for the pages converted to 16 bits once per call
    # (MKV_PREFILL_WORKSPACE=0 disables it, for tests and tuning)
    ws_n = lib.mkv_paged_prefill_workspace_bytes(num_seqs, total_q, num_heads, num_kv_heads, head_dim,
                                                 block_size, block_tables.shape[1], _DTYPES[query.dtype],
                                                 cache_code)
    if os.environ.get("MKV_PREFILL_WORKSPACE", "1") == "0":
        ws_n = 0
    ws = torch.empty(ws_n, dtype=torch.uint8, device=query.device) if ws_n else None
    with _on_device(dev):
        st = lib.mkv_paged_prefill(
            query.data_ptr(), query.stride(0), query.stride(1), _DTYPES[query.dtype],
            k_cache.data_ptr(), v_cache.data_ptr(), cache_code, kp, vp, kps, vps, num_blocks,
            block_size, block_tables.data_ptr(), _INDEX[block_tables.dtype], block_tables.stride(0),
            block_tables.shape[1], lens.data_ptr(), _INDEX[lens.dtype], cu.data_ptr(),
            _INDEX[cu.dtype], pos.data_ptr(), _INDEX[pos.dtype], num_seqs, total_q, num_heads,
            num_kv_heads, head_dim, float(scale), output.data_ptr(), output.stride(0),
            output.stride(1), ws.data_ptr() if ws is not None else None, ws_n, _stream(dev))
    _lib.check(fn, st)
    return output


def flash_attention_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            cu_seqlens: torch.Tensor, scale: float, num_heads: int,
                            num_kv_heads: int, head_dim: int,
                            max_seqlen: int | None = None) -> torch.Tensor:
    """Causal attention of each sequence over its own contiguous K/V (no KV cache):
    q (total_tokens, num_heads, head_dim), k/v (total_tokens, num_kv_heads, head_dim),
    sequence b owning rows [cu_seqlens[b], cu_seqlens[b+1]). Returns q's shape and dtype.
    Reference: flash_attention_prefill, attention.py:446-516 (kernel 336-443). Like the
    reference, it reads the longest sequence from cu_seqlens on the host unless
    `max_seqlen` (an upper bound, e.g. the context's max_seqlen_q) is given."""
    fn = "flash_attention_prefill"
    if q.dim() != 3 or q.shape[1] != num_heads or q.shape[2] != head_dim:
        raise ValueError(f"{fn}: q must be (total_tokens, {num_heads}, {head_dim}), got {tuple(q.shape)}")
    if q.dtype not in _FLOAT_IO:
        raise ValueError(f"{fn}: unsupported dtype {q.dtype}")
    dev = _require_cuda(fn, q, k, v, cu_seqlens)
    total = q.shape[0]
    if k.shape != (total, num_kv_heads, head_dim) or v.shape != k.shape:
        raise ValueError(f"{fn}: k/v must be ({total}, {num_kv_heads}, {head_dim})")
    if k.dtype != q.dtype:
        k = k.to(q.dtype)
    if v.dtype != q.dtype:
        v = v.to(q.dtype)
    q = q if q.stride(-1) == 1 and q.stride(1) % 8 == 0 and q.stride(0) % 8 == 0 else q.contiguous()
    k, v = _row_major_tokens(k), _row_major_tokens(v)
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    cu = _index_tensor(cu_seqlens.reshape(-1), fn, "cu_seqlens")
    num_seqs = cu.numel() - 1
    if total == 0 or num_seqs <= 0:
        return out
    if max_seqlen is None or max_seqlen <= 0:
        host = cu.cpu()
        max_seqlen = int((host[1:] - host[:-1]).max())
    max_seqlen = max(1, min(int(max_seqlen), total))
    lib = _lib.load()
    dt = _DTYPES[q.dtype]
    ws_n = lib.mkv_varlen_prefill_workspace_bytes(num_seqs, total, max_seqlen, num_kv_heads,
                                                  head_dim, dt)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=dev)
    with _on_device(dev):
        st = lib.mkv_varlen_prefill(
            q.data_ptr(), q.stride(0), q.stride(1), dt, k.data_ptr(), v.data_ptr(), k.stride(0),
            k.stride(1), v.stride(0), v.stride(1), cu.data_ptr(), _INDEX[cu.dtype], num_seqs, total,
            max_seqlen, num_heads, num_kv_heads, head_dim, float(scale), out.data_ptr(),
            out.stride(0), out.stride(1), ws.data_ptr(), ws_n, _stream(dev))
    _lib.check(fn, st)
    return out


# ---------------------------------------------------------------------------------- module
class Attention(nn.Module):
    """Attention layer with a paged KV cache (reference attention.py:1617-1807).

    The model runner injects `k_cache`/`v_cache` (per-layer views of one
    (2, L, num_blocks, block_size, KVH, D) allocation), `kv_cache_dtype`, and for the
    quantised modes the per-layer `k_scale`/`v_scale` (float32; shape (1,) initialised to
    the sentinel 1.0 for 'fp8_per_tensor', (num_blocks, block_size, KVH) for the
    per-(token, head) modes).
    `forward` appends the step's K/V at context.slot_mapping and, for a decode batch,
    returns (batch, num_heads * head_dim); a prefill, chunked-prefill or mixed batch
    attends through the paged cache (paged_attention_prefill for its prefill rows)."""

    def __init__(self, num_heads: int, head_dim: int, scale: float = 1.0,
                 num_kv_heads: int | None = None, block_size: int = 16):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads if num_kv_heads is not None else num_heads
        self.block_size = block_size
        self.k_cache = self.v_cache = torch.tensor([])
        self.kv_cache_dtype = "auto"
        self.k_scale = None
        self.v_scale = None

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        mode = self.kv_cache_dtype
        quant = mode != "auto"
        if mode not in ("auto", "fp8_per_tensor") + _PER_TOKEN_HEAD:
            raise NotImplementedError(f"kv_cache_dtype {mode!r} is not implemented")
        appended = False
        if k_cache.numel() > 0 and v_cache.numel() > 0 and context.slot_mapping is not None:
            appended = True
            if k.dim() == 4:
                b, n, kvh, d = k.shape
                k, v = k.reshape(b * n, kvh, d), v.reshape(b * n, kvh, d)
            if mode == "int8_per_token_head":
                store_kvcache_int8(k, v, k_cache, v_cache, self.k_scale, self.v_scale,
                                   context.slot_mapping, self.block_size)
            elif quant:
                store_kvcache_fp8(k, v, k_cache, v_cache, self.k_scale, self.v_scale,
                                  context.slot_mapping, self.block_size, mode)
            else:
                store_kvcache(k, v, k_cache, v_cache, context.slot_mapping, self.block_size)
        scale = self.scale / (self.head_dim ** 0.5)
        if context.is_prefill:
            if getattr(context, "is_full_prefill", False):
                # every sequence is a whole prompt: attend over the step's own q/k/v, as the
                # reference does (attention.py:1771), which also serves the runner's
                # warm-up before the KV cache exists
                if context.cu_seqlens_q is None:
                    raise ValueError("cu_seqlens_q must be provided for varlen attention")
                if k.dim() == 4:
                    b, n, kvh, d = k.shape
                    k, v = k.reshape(b * n, kvh, d), v.reshape(b * n, kvh, d)
                o = flash_attention_prefill(q, k, v, context.cu_seqlens_q, scale, self.num_heads,
                                            self.num_kv_heads, self.head_dim,
                                            getattr(context, "max_seqlen_q", 0) or None)
                return o.reshape(o.shape[0], self.num_heads * self.head_dim)
            return self._prefill(q, k_cache, v_cache, context, scale, mode, quant)
        # The append (if any) was the last kernel launched and writes only the pages (and
        # scales): the decode's prologue may overlap it. Without an append the previous
        # kernel may have produced q, so no overlap.
        overlap = appended
        if quant:
            o = paged_attention_decode_quantized(
                q, k_cache, v_cache, self.k_scale, self.v_scale, context.block_tables,
                context.context_lens, scale, self.num_heads, self.num_kv_heads, self.head_dim,
                self.block_size, self.kv_cache_dtype, overlap_previous=overlap)
        else:
            o = paged_attention_decode(
                q, k_cache, v_cache, context.block_tables, context.context_lens, scale,
                self.num_heads, self.num_kv_heads, self.head_dim, self.block_size,
                overlap_previous=overlap)
        return o.reshape(o.shape[0], self.num_heads * self.head_dim)

    def _decode_rows(self, q, k_cache, v_cache, block_tables, context_lens, scale, mode, quant):
        if quant:
            return paged_attention_decode_quantized(
                q, k_cache, v_cache, self.k_scale, self.v_scale, block_tables, context_lens,
                scale, self.num_heads, self.num_kv_heads, self.head_dim, self.block_size, mode)
        return paged_attention_decode(q, k_cache, v_cache, block_tables, context_lens, scale,
                                      self.num_heads, self.num_kv_heads, self.head_dim,
                                      self.block_size)

    def _prefill(self, q, k_cache, v_cache, context, scale, mode, quant):
        """Chunked prefill, extend and mixed batches (context.is_full_prefill False) read the
        whole visible context from the paged cache (the step's K/V were appended just
        before), as attention.py:1695-1770 does; a mixed batch's decode rows go through the decode
        kernels (1711-1760). Quantised caches are dequantised in the kernel (the reference
        raises NotImplementedError there, 1702-1708)."""
        if context.cu_seqlens_q is None:
            raise ValueError("cu_seqlens_q must be provided for varlen attention")
        if context.positions is None or context.context_lens is None or context.block_tables is None:
            raise ValueError("paged prefill requires positions, context_lens, and block_tables")
        ks, vs = (self.k_scale, self.v_scale) if quant else (None, None)
        split = getattr(context, "mixed_attention_split", None)
        if split is not None and split.decode_token_indices and split.prefill_token_indices:
            o = torch.empty_like(q)
            di, ds = split.decode_token_indices_tensor, split.decode_seq_indices_tensor
            o.index_copy_(0, di, self._decode_rows(
                q.index_select(0, di), k_cache, v_cache, context.block_tables.index_select(0, ds),
                context.context_lens.index_select(0, ds), scale, mode, quant))
            pi, ps = split.prefill_token_indices_tensor, split.prefill_seq_indices_tensor
            o.index_copy_(0, pi, paged_attention_prefill(
                q.index_select(0, pi), k_cache, v_cache, context.block_tables.index_select(0, ps),
                context.context_lens.index_select(0, ps), split.prefill_cu_seqlens_q_tensor,
                context.positions.index_select(0, pi), scale, self.num_heads, self.num_kv_heads,
                self.head_dim, self.block_size, ks, vs, mode))
            return o.reshape(o.shape[0], self.num_heads * self.head_dim)
        o = paged_attention_prefill(q, k_cache, v_cache, context.block_tables, context.context_lens,
                                    context.cu_seqlens_q, context.positions, scale, self.num_heads,
                                    self.num_kv_heads, self.head_dim, self.block_size, ks, vs, mode)
        return o.reshape(o.shape[0], self.num_heads * self.head_dim)
