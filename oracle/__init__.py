"""CPU oracle for the paged KV-cache hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU with torch, the reference algorithm of
heart1128/mini-kvllm for the KV append (bf16/fp16/fp32, FP8 E4M3 per-tensor, FP8 and
INT8 per-(token, head)), the paged-attention decode, the chunked-prefill / extend
attention over the paged cache, and the tensor-parallel all-reduce + residual add +
RMSNorm that ends each projection. It is the checker, never the product: only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import it.
The CUDA library (libmkv.so) never calls into it and has no CPU fallback.

Parity pin: tests/golden/ holds fixtures produced by running the reference's own
functions (src/myvllm/layers/attention.py under the Triton interpreter, and
benchmark_decoding.py's decode_torch_optimized) on seeded inputs, together with
the script that made them; tests/test_oracle_golden.py checks this oracle against
them. See kv_oracle.py for the per-function reference citations.
"""
from .kv_oracle import (  # noqa: F401
    FP8_E4M3_MAX,
    allreduce_residual_rmsnorm_ref,
    INT8_MAX,
    INT8_MIN,
    decode_torch_optimized,
    e4m3_encode_reference,
    fp8_scale_ref,
    paged_decode_ref,
    paged_prefill_ref,
    per_token_head_scales_ref,
    quantize_fp8_ref,
    quantize_int8_ref,
    store_kvcache_fp8_ref,
    store_kvcache_quant_per_token_head_ref,
    store_kvcache_ref,
    varlen_prefill_ref,
)
