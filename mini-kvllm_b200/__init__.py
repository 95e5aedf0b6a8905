"""B200-native paged KV-cache hot path of mini-kvllm: KV append (bf16/fp16/fp32 and
FP8 E4M3 per-tensor) and paged-attention decode, as sm_100a CUDA kernels behind the
C ABI of libmkv.so (include/mkv.h), with the reference's Python call signatures.

The directory name contains a hyphen, so import it with importlib:
    mkv = importlib.import_module("mini-kvllm_b200")
    from importlib import import_module
    attn = import_module("mini-kvllm_b200.layers.attention")
"""
from . import _lib
from ._lib import LIB_PATH, MkvError, load
from .layers.attention import (
    Attention,
    flash_attention_prefill,
    paged_attention_decode,
    paged_attention_decode_quantized,
    store_kvcache,
    store_kvcache_fp8,
)
from .utils.context import Context, get_context, reset_context, set_context

__all__ = [
    "Attention", "Context", "LIB_PATH", "MkvError", "flash_attention_prefill", "get_context", "load",
    "paged_attention_decode", "paged_attention_decode_quantized", "reset_context",
    "set_context", "store_kvcache", "store_kvcache_fp8",
]
