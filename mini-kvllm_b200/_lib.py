"""ctypes binding of libmkv.so, the C-ABI CUDA library declared in include/mkv.h.

The library is loaded from this package directory. There is no fallback: when the
library is missing, `load()` raises with the command that builds it, so a product
path can never silently run anything but the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libmkv.so")

# Constants mirrored from include/mkv.h.
DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_FP8_E4M3, DTYPE_INT8 = 0, 1, 2, 3, 4
INDEX_I32, INDEX_I64 = 0, 1
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA = 0, 1, 2, 3, 4
FP8_CALIB_WORK_BYTES = 16
DECODE_OVERLAP_PREVIOUS = 2
NOALLOC_SCRATCH_BYTES = 16 << 20
AR_MAX_RANKS, AR_MAX_BLOCKS, IPC_HANDLE_BYTES = 8, 128, 64
AR_FLAG_BYTES = AR_MAX_BLOCKS * AR_MAX_RANKS * 4

# Every symbol include/mkv.h declares, with (restype, argtypes).
_p, _i32, _i64, _f32, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
_cstr = ctypes.c_char_p
SIGNATURES: dict[str, tuple] = {
    "mkv_version": (_cstr, []),
    "mkv_source_hash": (_cstr, []),
    "mkv_status_string": (_cstr, [ctypes.c_int]),
    "mkv_last_error": (_cstr, []),
    "mkv_store_kvcache": (ctypes.c_int, [
        _p, _p, _i64, _i64, _i64, _i64, _p, _p, _i64, _i32, _p, _i32, _i64, _i32, _i32, _i32, _p, _p]),
    "mkv_calibrate_fp8_scales": (ctypes.c_int, [
        _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _p, _p, _p, _p]),
    "mkv_store_kvcache_fp8": (ctypes.c_int, [
        _p, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i32, _p, _i32, _i64, _i32, _i32, _i32, _p, _p]),
    "mkv_store_kvcache_fp8_calibrating": (ctypes.c_int, [
        _p, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i32, _p, _i32, _i64, _i32, _i32, _i32, _p, _p,
        _p]),
    "mkv_store_kvcache_quant_per_token_head": (ctypes.c_int, [
        _p, _p, _i64, _i64, _i64, _i64, _p, _p, _i32, _p, _p, _i64, _i32, _p, _i32, _i64, _i32, _i32,
        _i32, _p, _p]),
    "mkv_paged_decode_num_splits": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "mkv_paged_decode_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "mkv_paged_decode": (ctypes.c_int, [
        _p, _i64, _i64, _i32, _p, _p, _i32, _i64, _i32, _p, _i32, _i64, _i32, _p, _i32,
        _i32, _i32, _i32, _i32, _f32, _p, _i64, _i64, _p, _sz, _i32, _p, _p]),
    "mkv_paged_decode_noalloc": (ctypes.c_int, [
        _p, _i64, _i64, _i32, _p, _p, _i32, _i64, _i32, _p, _i32, _i64, _i32, _p, _i32,
        _i32, _i32, _i32, _i32, _f32, _p, _i64, _i64, _i32, _p, _p]),
    "mkv_paged_decode_ex": (ctypes.c_int, [
        _p, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _p, _p, _i64, _i32, _p, _i32, _i64, _i32, _p, _i32,
        _i32, _i32, _i32, _i32, _f32, _p, _i64, _i64, _p, _sz, _p, _sz, _i32, ctypes.c_uint32, _p, _p]),
    "mkv_paged_decode_counter_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "mkv_paged_decode_quant_per_token_head": (ctypes.c_int, [
        _p, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _i64, _i32, _p, _i32, _i64, _i32, _p, _i32,
        _i32, _i32, _i32, _i32, _f32, _p, _i64, _i64, _p, _sz, _i32, _p, _p]),
    "mkv_paged_prefill": (ctypes.c_int, [
        _p, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _p, _p, _i64, _i32, _p, _i32, _i64, _i32, _p, _i32,
        _p, _i32, _p, _i32, _i32, _i64, _i32, _i32, _i32, _f32, _p, _i64, _i64, _p, _sz, _p]),
    "mkv_paged_prefill_workspace_bytes": (_sz, [_i32, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "mkv_varlen_prefill_workspace_bytes": (_sz, [_i32, _i64, _i32, _i32, _i32, _i32]),
    "mkv_varlen_prefill": (ctypes.c_int, [
        _p, _i64, _i64, _i32, _p, _p, _i64, _i64, _i64, _i64, _p, _i32, _i32, _i64, _i32, _i32, _i32, _i32,
        _f32, _p, _i64, _i64, _p, _sz, _p]),
    "mkv_allreduce_residual_rmsnorm": (ctypes.c_int, [
        _p, _p, _i64, _p, _i32, _i32, _p, _p, _p, _p, _p, _i64, _i32, _i32, _f32, _p, _i64, _p]),
    "mkv_decode_metadata": (ctypes.c_int, [_p, _i32, _i32, _i32, _p, _p, _p]),
    "mkv_ipc_alloc": (ctypes.c_int, [_sz, ctypes.POINTER(_p), _p]),
    "mkv_ipc_free": (ctypes.c_int, [_p]),
    "mkv_ipc_open": (ctypes.c_int, [_p, ctypes.POINTER(_p)]),
    "mkv_ipc_close": (ctypes.c_int, [_p]),
    "mkv_paged_decode_fp8": (ctypes.c_int, [
        _p, _i64, _i64, _i32, _p, _p, _p, _p, _i64, _i32, _p, _i32, _i64, _i32, _p, _i32,
        _i32, _i32, _i32, _i32, _f32, _p, _i64, _i64, _p, _sz, _i32, _p, _p]),
}


class MkvError(RuntimeError):
    """A libmkv entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        self.status = status
        super().__init__(f"{fn} failed with status {status}: {message}")


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Returns the loaded library, loading it (once) on first use."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libmkv.so is not built ({LIB_PATH} missing). Build it with "
                    f"`python {os.path.join(PKG_DIR, 'build.py')}` (needs nvcc 12.9+).")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def source_hash() -> str:
    """Hash of the sources the loaded libmkv.so was built from (see build.py)."""
    return load().mkv_source_hash().decode()


def check(fn: str, status: int) -> None:
    """Raises MkvError (ValueError-like statuses included) for a non-zero status."""
    if status != OK:
        msg = load().mkv_last_error().decode(errors="replace")
        if status in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE):
            raise ValueError(f"{fn}: {msg}")
        raise MkvError(fn, status, msg)
