/*
 * mkv.h — C ABI of the B200 paged KV-cache library (libmkv.so).
 *
 * The library implements the two halves of mini-kvllm's per-layer attention hot path:
 *   - the KV append (store new K/V rows into block-table pages, optionally
 *     quantised to FP8 E4M3 with a per-tensor scale), and
 *   - the paged-attention decode (one query token per sequence, GQA head
 *     grouping, FP8 dequantisation fused into the page loads, online softmax,
 *     split-KV partitioning with an in-kernel merge).
 *
 * Every entry point takes plain device pointers, element strides and sizes, and a
 * CUDA stream passed as `void*` (a `cudaStream_t`; NULL = legacy default stream).
 * Nothing here allocates device memory: the decode's split-KV scratch and the FP8
 * calibration words are caller-provided workspaces. All launches are asynchronous
 * on `stream` and contain no host synchronisation, so they can be captured in a
 * CUDA graph.
 *
 * Each function returns MKV_OK (0) or an error code; mkv_last_error() then holds a
 * message for the calling thread. Argument errors are detected on the host before
 * any CUDA call. Index values read on the device (slots, block-table entries) are
 * bounds-checked in the kernels: an out-of-range entry is skipped, never
 * dereferenced, and counted in the optional `invalid_count` word.
 *
 * Tensor layouts (row-major, innermost last):
 *   key/value     (num_tokens, num_kv_heads, head_dim)   strides given per call
 *   k/v cache     (num_blocks, block_size, num_kv_heads, head_dim)   contiguous
 *   slot_mapping  (num_tokens,)              int32 or int64, -1 = skip this token
 *   query / out   (num_seqs, num_heads, head_dim)        strides given per call
 *   block_tables  (num_seqs, max_num_blocks) int32 or int64, -1 = no page
 *   context_lens  (num_seqs,)                int32 or int64
 *   k/v scale     one float32 each (per-tensor FP8 scale)
 *
 * Reference: heart1128/mini-kvllm, src/myvllm/layers/attention.py. Each entry
 * point below names the reference function it replaces.
 */
#ifndef MKV_H_
#define MKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Symbol visibility: the library is built with hidden visibility; only these are exported. */
#if defined(__GNUC__)
#define MKV_API __attribute__((visibility("default")))
#else
#define MKV_API
#endif

/* Element types (also the dtype of query/out and key/value). */
#define MKV_DTYPE_F32 0
#define MKV_DTYPE_F16 1
#define MKV_DTYPE_BF16 2
#define MKV_DTYPE_FP8_E4M3 3
#define MKV_DTYPE_INT8 4

/* Integer index types for slot_mapping / block_tables / context_lens. */
#define MKV_INDEX_I32 0
#define MKV_INDEX_I64 1

/* Status codes. */
#define MKV_OK 0
#define MKV_ERR_INVALID_ARGUMENT 1
#define MKV_ERR_UNSUPPORTED 2
#define MKV_ERR_WORKSPACE 3
#define MKV_ERR_CUDA 4

/* Library version string ("major.minor.patch"). */
MKV_API const char* mkv_version(void);

/* 16 hex digits identifying the sources and compiler flags the library was built from,
   so that every measurement can name the exact binary it ran. No reference counterpart. */
MKV_API const char* mkv_source_hash(void);

/* Human-readable name of a status code. */
MKV_API const char* mkv_status_string(int status);

/* Message describing the last error returned on the calling thread ("" if none). */
MKV_API const char* mkv_last_error(void);

/*
 * KV append, same dtype in and out (bf16, fp16 or fp32).
 * Replaces store_kvcache (attention.py:67-108) and its kernel
 * store_kvcache_kernel (attention.py:7-64):
 *     k_cache.view(-1, KVH, D)[slot_mapping[t]] = key[t]   (same for value)
 * Tokens whose slot is negative are skipped (the reference skips slot -1,
 * attention.py:29-30). Slots >= num_blocks*block_size are skipped and counted in
 * *invalid_count when that pointer is non-NULL (device int32, accumulated).
 * Strides are in elements; head_dim must be contiguous.
 */
MKV_API int mkv_store_kvcache(const void* key, const void* value,
                      int64_t key_stride_token, int64_t key_stride_head,
                      int64_t value_stride_token, int64_t value_stride_head,
                      void* k_cache, void* v_cache,
                      int64_t num_blocks, int32_t block_size,
                      const void* slot_mapping, int32_t slot_index_type,
                      int64_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                      int32_t dtype, int32_t* invalid_count, void* stream);

/*
 * Device-side, sentinel-aware per-tensor FP8 calibration of the K and V scales.
 * Replaces the host block of store_kvcache_fp8 (attention.py:315-323):
 *     if scale == 1.0:  scale = dtype(max(amax(|x|), dtype(1e-8)) * fp32(1/448))
 * i.e. the value torch produces for `x.abs().amax().clamp(min=1e-8) / 448.0` on a
 * CUDA tensor of the key dtype (bf16/fp16/fp32; torch divides by a Python scalar
 * as a multiplication by its float32 reciprocal), stored as float32. A scale that
 * already differs from 1.0 is left untouched (the scale is frozen after the first
 * calibration). The amax covers every token of key/value, including tokens whose
 * slot is -1, exactly as the reference's key.abs().amax().
 * `work` is a caller-provided device buffer of MKV_FP8_CALIB_WORK_BYTES bytes that
 * must be zero before the first call; every call leaves it zero again. Calls that
 * share one `work` buffer must be ordered on one stream.
 */
#define MKV_FP8_CALIB_WORK_BYTES 16
MKV_API int mkv_calibrate_fp8_scales(const void* key, const void* value,
                             int64_t key_stride_token, int64_t key_stride_head,
                             int64_t value_stride_token, int64_t value_stride_head,
                             int64_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                             int32_t dtype, float* k_scale, float* v_scale,
                             void* work, void* stream);

/*
 * KV append with FP8 E4M3 quantisation, per-tensor scales read on the device.
 * Replaces the per-tensor branch of store_kvcache_fp8_kernel
 * (attention.py:118-191, 182-191):
 *     cache[slot] = e4m3(clamp(float(x) / scale, -448, 448))
 * with IEEE division and round-to-nearest-even conversion. Slot rules as in
 * mkv_store_kvcache. head_dim must be a multiple of 16.
 */
MKV_API int mkv_store_kvcache_fp8(const void* key, const void* value,
                          int64_t key_stride_token, int64_t key_stride_head,
                          int64_t value_stride_token, int64_t value_stride_head,
                          void* k_cache, void* v_cache,
                          const float* k_scale, const float* v_scale,
                          int64_t num_blocks, int32_t block_size,
                          const void* slot_mapping, int32_t slot_index_type,
                          int64_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                          int32_t dtype, int32_t* invalid_count, void* stream);

/*
 * The whole of store_kvcache_fp8's per-tensor path in one launch (attention.py:281-333):
 * the calibration of mkv_calibrate_fp8_scales (315-323) for each scale that still holds
 * the sentinel 1.0, then the quantising store of mkv_store_kvcache_fp8 (118-191) with
 * the scales as they then are. Results are bit-identical to those two calls in a row.
 * In the steady state (both scales calibrated) the kernel reads the scales and stores;
 * while a scale is the sentinel, every CTA adds its share of the batch's amax into
 * `calib_work` and the last CTA to finish writes the scale(s) and quantises the batch.
 * No CTA ever waits for another. `calib_work`: MKV_FP8_CALIB_WORK_BYTES of device
 * memory, zero before the first call and left zero by every call; calls sharing it
 * must be ordered on one stream. calib_work = NULL quantises with the scales as they
 * are (no calibration), like mkv_store_kvcache_fp8 (which takes the same kernel).
 */
MKV_API int mkv_store_kvcache_fp8_calibrating(
    const void* key, const void* value, int64_t key_stride_token, int64_t key_stride_head,
    int64_t value_stride_token, int64_t value_stride_head, void* k_cache, void* v_cache,
    float* k_scale, float* v_scale, int64_t num_blocks, int32_t block_size,
    const void* slot_mapping, int32_t slot_index_type, int64_t num_tokens, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype, void* calib_work, int32_t* invalid_count, void* stream);

/*
 * KV append with a dynamic scale per (token, kv head) row, into an FP8 E4M3 or INT8
 * cache (cache_dtype MKV_DTYPE_FP8_E4M3 or MKV_DTYPE_INT8). Replaces store_kvcache_fp8
 * with kv_cache_dtype "fp8_per_token_head" (attention.py:281-333 with the kernel
 * store_kvcache_fp8_kernel, PER_TOKEN_HEAD=1, attention.py:118-191) and store_kvcache_int8
 * (attention.py:195-278). For each stored row, with amax = max |x| over head_dim:
 *   FP8:  scale = amax > 0 ? amax / 448 : 1;  byte = e4m3(clamp(x / scale, -448, 448))
 *   INT8: scale = max(amax / 127, 1e-6);      q = x * (1 / scale), rounded half away
 *         from zero, clamped to [-128, 127]
 * (IEEE float32 division; a row holding NaN gets scale 1 (FP8) or 1e-6 (INT8)).
 * k_scales/v_scales are float32 (num_blocks, block_size, num_kv_heads); the row's scale
 * is written at its slot. Slot rules as in mkv_store_kvcache. head_dim must be a
 * multiple of 16 and at most 512; caches 16-byte aligned.
 */
MKV_API int mkv_store_kvcache_quant_per_token_head(
    const void* key, const void* value, int64_t key_stride_token, int64_t key_stride_head,
    int64_t value_stride_token, int64_t value_stride_head, void* k_cache, void* v_cache,
    int32_t cache_dtype, float* k_scales, float* v_scales, int64_t num_blocks,
    int32_t block_size, const void* slot_mapping, int32_t slot_index_type, int64_t num_tokens,
    int32_t num_kv_heads, int32_t head_dim, int32_t dtype, int32_t* invalid_count, void* stream);

/*
 * Split count the decode uses for this shape when num_splits = 0 (auto). Returns 0
 * when auto means the balanced schedule: the grid is the kernel's resident CTAs and
 * each takes an equal share of all (sequence, kv head) token tiles, computed on the
 * device from context_lens, so long units are split where CTA shares end. A positive
 * value is a fixed split count (only for shapes beyond the balanced schedule's
 * 64-bit work-item arithmetic). Host-only; depends on shapes, never on device data.
 */
MKV_API int32_t mkv_paged_decode_num_splits(int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                    int32_t head_dim, int32_t block_size, int32_t max_num_blocks);

/*
 * Bytes of workspace the decode needs for this shape and split count.
 * num_splits = 0 (auto, balanced schedule): 2 partial slots per resident CTA
 * (at most 148 x 4 CTAs) of min(H / KVH, 16) heads x (head_dim + 2) floats, plus one
 * arrival counter per (sequence, kv head, head group); it does not grow with the
 * context length. num_splits > 0: one partial per (sequence, head, split) plus the
 * counters; 0 when num_splits = 1.
 */
MKV_API size_t mkv_paged_decode_workspace_bytes(int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                        int32_t head_dim, int32_t block_size,
                                        int32_t max_num_blocks, int32_t num_splits);

/*
 * Paged-attention decode over a bf16 / fp16 / fp32 cache.
 * Replaces paged_attention_decode (attention.py:895-950) and its kernel
 * paged_attention_decode_kernel (attention.py:517-646):
 *     out[b, h] = softmax_t(scale * q[b, h] . K[b, kvh(h), t]) V[b, kvh(h), t]
 * over t < min(context_lens[b], max_num_blocks*block_size), with page
 * block_tables[b, t / block_size] and row t % block_size; kvh(h) = h / (H / KVH).
 * Tokens on a page entry that is -1 (or outside [0, num_blocks)) are skipped,
 * as in the reference. A sequence with no visible token yields NaN (0/0), as in
 * the reference. out has query's dtype. workspace may be NULL when
 * mkv_paged_decode_workspace_bytes(...) is 0.
 */
MKV_API int mkv_paged_decode(const void* query, int64_t q_stride_seq, int64_t q_stride_head, int32_t q_dtype,
                     const void* k_cache, const void* v_cache, int32_t cache_dtype,
                     int64_t num_blocks, int32_t block_size,
                     const void* block_tables, int32_t block_table_index_type,
                     int64_t block_table_stride_seq, int32_t max_num_blocks,
                     const void* context_lens, int32_t context_lens_index_type,
                     int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                     float scale, void* out, int64_t out_stride_seq, int64_t out_stride_head,
                     void* workspace, size_t workspace_bytes, int32_t num_splits,
                     int32_t* invalid_count, void* stream);

/*
 * Paged-attention decode over an FP8 E4M3 cache with per-tensor scales
 * (device float32 each). Replaces paged_attention_decode_quantized
 * (attention.py:1213-1268) for kv_cache_dtype "fp8_per_tensor", i.e.
 * paged_attention_decode_fp8_kernel with PER_TOKEN_HEAD=0 (attention.py:953-1121):
 * K = float(k_fp8) * k_scale and V = float(v_fp8) * v_scale, dequantised as the
 * pages are loaded. Other arguments as in mkv_paged_decode.
 */
MKV_API int mkv_paged_decode_fp8(const void* query, int64_t q_stride_seq, int64_t q_stride_head, int32_t q_dtype,
                         const void* k_cache, const void* v_cache,
                         const float* k_scale, const float* v_scale,
                         int64_t num_blocks, int32_t block_size,
                         const void* block_tables, int32_t block_table_index_type,
                         int64_t block_table_stride_seq, int32_t max_num_blocks,
                         const void* context_lens, int32_t context_lens_index_type,
                         int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                         float scale, void* out, int64_t out_stride_seq, int64_t out_stride_head,
                         void* workspace, size_t workspace_bytes, int32_t num_splits,
                         int32_t* invalid_count, void* stream);

/*
 * Paged-attention decode over an FP8 E4M3 or INT8 cache (cache_dtype) with one scale
 * per (page, row, kv head): K = float(k) * k_scales[page, row, kvh], V likewise, with
 * k_scales/v_scales float32 (num_blocks, block_size, num_kv_heads) as written by
 * mkv_store_kvcache_quant_per_token_head. Replaces paged_attention_decode_quantized for
 * kv_cache_dtype "fp8_per_token_head" and "int8_per_token_head" (attention.py:1213-1268;
 * kernels paged_attention_decode_quantized_tile_kernel, attention.py:1124-1210, and
 * paged_attention_decode_fp8_kernel with PER_TOKEN_HEAD=1, attention.py:953-1121).
 * A -1 (or out-of-range) page inside a context is skipped, as the reference's FP8
 * kernel does (its tile kernel, used for head_dim <= 128, instead scores such tokens
 * 0 against a zero V). Other arguments as in mkv_paged_decode; the workspace size is
 * mkv_paged_decode_workspace_bytes(...).
 */
MKV_API int mkv_paged_decode_quant_per_token_head(
    const void* query, int64_t q_stride_seq, int64_t q_stride_head, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t cache_dtype, const float* k_scales,
    const float* v_scales, int64_t num_blocks, int32_t block_size, const void* block_tables,
    int32_t block_table_index_type, int64_t block_table_stride_seq, int32_t max_num_blocks,
    const void* context_lens, int32_t context_lens_index_type, int32_t num_seqs,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float scale, void* out,
    int64_t out_stride_seq, int64_t out_stride_head, void* workspace, size_t workspace_bytes,
    int32_t num_splits, int32_t* invalid_count, void* stream);

/*
 * Chunked-prefill / extend attention over the paged cache. Replaces
 * paged_attention_prefill_triton (attention.py:852-892; kernel 704-849) and
 * paged_attention_prefill_torch (649-701). query (total_q, num_heads, head_dim) holds the
 * new tokens of every sequence, sequence b owning rows [cu_seqlens_q[b], cu_seqlens_q[b+1]);
 * row q at absolute position positions[q] attends to the cached tokens
 * t < min(context_lens[b], positions[q] + 1) on pages block_tables[b, t / block_size]
 * (its own K/V must already be appended). -1 and out-of-range pages are skipped (not
 * counted); a row that sees no token gives NaN. out has query's layout and dtype.
 * Caches: the query dtype (bf16, f16, f32), or 8-bit with scales dequantised on load
 * (not in the reference, whose TODO asks for it): FP8_E4M3 with per-tensor k_scale /
 * v_scale, or FP8_E4M3 / INT8 with per-(page, row, kv head) k_scales / v_scales (pass
 * the other pair as NULL). Tensor cores for bf16/f16 queries with head_dim 64 or 128;
 * CUDA cores otherwise (head_dim a multiple of 16, at most 256).
 *
 * workspace (16-byte aligned) may be NULL. With 8-bit caches and long chunks, a
 * workspace of at least mkv_paged_prefill_workspace_bytes(...) lets the call convert
 * each visible page to 16 bits once, into the workspace, and run the 16-bit tensor-core
 * kernel over it; without one, the 8-bit tiles are converted inside the attention
 * kernel, once per query block. Both compute the same attention. Its contents on entry
 * do not matter.
 */
MKV_API int mkv_paged_prefill(
    const void* query, int64_t q_stride_token, int64_t q_stride_head, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t cache_dtype, const float* k_scale,
    const float* v_scale, const float* k_scales, const float* v_scales, int64_t num_blocks,
    int32_t block_size, const void* block_tables, int32_t block_table_index_type,
    int64_t block_table_stride_seq, int32_t max_num_blocks, const void* context_lens,
    int32_t context_lens_index_type, const void* cu_seqlens_q, int32_t cu_seqlens_index_type,
    const void* positions, int32_t positions_index_type, int32_t num_seqs, int64_t total_q,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float scale, void* out,
    int64_t out_stride_token, int64_t out_stride_head, void* workspace, size_t workspace_bytes,
    void* stream);

/*
 * Workspace bytes mkv_paged_prefill uses for the given shape: 2 x num_seqs x
 * max_num_blocks x block_size x num_kv_heads x head_dim 16-bit values (the visible pages
 * converted to the query dtype) when the cache is 8-bit (FP8_E4M3 or INT8), the query
 * bf16 or f16, head_dim 128, num_heads / num_kv_heads <= 128, block_size a power of two
 * >= 8, the sequences hold at least 512 query rows (query tokens x GQA group) on average,
 * and the total is at most 1 GiB; 0 otherwise (no workspace is used). Host-only: reads
 * no device memory.
 */
MKV_API size_t mkv_paged_prefill_workspace_bytes(int32_t num_seqs, int64_t total_q,
                                                 int32_t num_heads, int32_t num_kv_heads,
                                                 int32_t head_dim, int32_t block_size,
                                                 int32_t max_num_blocks, int32_t q_dtype,
                                                 int32_t cache_dtype);

/*
 * Causal attention of variable-length sequences over their own contiguous K/V: the
 * reference's flash_attention_prefill (attention.py:446-516, kernel 336-443), which
 * Attention.forward takes when the batch is whole prompts (context.is_full_prefill,
 * attention.py:1771) and the model runner's warm-up takes before a KV cache exists
 * (model_runner.py:193-200). Sequence b owns rows [cu_seqlens[b], cu_seqlens[b+1]) of
 * query (total_tokens, num_heads, head_dim) and of key/value (total_tokens, num_kv_heads,
 * head_dim); row i at position t = i - cu_seqlens[b] attends to that sequence's tokens
 * 0..t, kv head of query head h being h / (num_heads / num_kv_heads); out has the query's
 * shape and dtype (f32/f16/bf16, key/value the same dtype, head_dim rows 16-byte aligned).
 * max_seqlen must bound every sequence's length. The K/V rows are packed into 128-row
 * pages of the workspace (mkv_varlen_prefill_workspace_bytes, 256-byte aligned) and
 * mkv_paged_prefill runs over them.
 */
MKV_API size_t mkv_varlen_prefill_workspace_bytes(int32_t num_seqs, int64_t total_tokens,
                                                  int32_t max_seqlen, int32_t num_kv_heads,
                                                  int32_t head_dim, int32_t dtype);
MKV_API int mkv_varlen_prefill(
    const void* query, int64_t q_stride_token, int64_t q_stride_head, int32_t dtype,
    const void* key, const void* value, int64_t key_stride_token, int64_t key_stride_head,
    int64_t value_stride_token, int64_t value_stride_head, const void* cu_seqlens,
    int32_t cu_seqlens_index_type, int32_t num_seqs, int64_t total_tokens, int32_t max_seqlen,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float scale, void* out,
    int64_t out_stride_token, int64_t out_stride_head, void* workspace, size_t workspace_bytes,
    void* stream);

/*
 * Every decode mode behind one entry point, with launch options. The arguments mean
 * what they mean for mkv_paged_decode; the cache mode follows from cache_dtype and the
 * scale pointers: an FP8_E4M3 cache with k_scale/v_scale (one float32 each) is the
 * per-tensor mode of mkv_paged_decode_fp8; an FP8_E4M3 or INT8 cache with
 * k_scales/v_scales (num_blocks, block_size, num_kv_heads) is the per-(token, head)
 * mode of mkv_paged_decode_quant_per_token_head; no scales is mkv_paged_decode.
 * No reference counterpart (the reference launches one Triton kernel per mode).
 * counters (optional): a caller-kept buffer of at least mkv_paged_decode_counter_bytes(...)
 *   bytes for the split merge's arrival counters, all zero before its first use and
 *   used for nothing else. Every decode leaves the counters it touched at zero, so the
 *   buffer can serve all decodes that are ordered on one stream, whatever their shapes,
 *   and the call then issues no clearing memset (with counters NULL they live in the
 *   workspace and are cleared with one cudaMemsetAsync per call). The workspace size
 *   stays mkv_paged_decode_workspace_bytes(...); its counter part is then unused.
 * flags (bitwise or):
 *   MKV_DECODE_OVERLAP_PREVIOUS  programmatic dependent launch: the decode may start
 *       while the previous kernel on the stream still runs. Its prologue (the
 *       schedule's scan of context_lens, the block-table slice, the query rows) then
 *       overlaps that kernel, and it reads K/V pages (and per-token scales) only after
 *       that kernel has completed. Pass it only when that previous kernel writes none of
 *       query, block_tables and context_lens, e.g. when it is this library's KV append
 *       of the same step (whose kernels let a dependent start early).
 */
#define MKV_DECODE_OVERLAP_PREVIOUS 2u
MKV_API size_t mkv_paged_decode_counter_bytes(int32_t num_seqs, int32_t num_heads,
                                              int32_t num_kv_heads, int32_t head_dim,
                                              int32_t block_size, int32_t max_num_blocks,
                                              int32_t num_splits);
MKV_API int mkv_paged_decode_ex(
    const void* query, int64_t q_stride_seq, int64_t q_stride_head, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t cache_dtype, const float* k_scale,
    const float* v_scale, const float* k_scales, const float* v_scales, int64_t num_blocks,
    int32_t block_size, const void* block_tables, int32_t block_table_index_type,
    int64_t block_table_stride_seq, int32_t max_num_blocks, const void* context_lens,
    int32_t context_lens_index_type, int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, float scale, void* out, int64_t out_stride_seq, int64_t out_stride_head,
    void* workspace, size_t workspace_bytes, uint32_t* counters, size_t counters_bytes,
    int32_t num_splits, uint32_t flags, int32_t* invalid_count, void* stream);

/*
 * Paged-attention decode that allocates nothing and needs no workspace argument.
 * This entry point has no counterpart in the reference; it exists for callers that
 * cannot allocate device memory on their own: a host runtime that reserves all device
 * memory up front and hands out no temporary buffers, a real-time serving loop where
 * the device synchronisation of cudaMalloc is not allowed, or a foreign-language caller
 * (cgo, JNI, a C application) that holds device pointers from another runtime but has
 * no device allocator to create the decode workspace.
 *
 * It computes exactly what mkv_paged_decode computes (same arguments, minus the
 * workspace; bf16/fp16/fp32 caches only). The split-KV scratch lives in an array built
 * into the library, MKV_NOALLOC_SCRATCH_BYTES (16 MiB) per device, which every GPU
 * that loads the library keeps until the process exits. A shape whose split scratch
 * (mkv_paged_decode_workspace_bytes with the same num_splits) exceeds that size is
 * rejected with MKV_ERR_WORKSPACE; num_splits = 1 needs no scratch at all.
 * The first call in a CUDA context looks up the array's device address in that context
 * (cudaGetSymbolAddress, with the caller's device current) and caches it for that
 * context only, keyed on the context's unique ID (cuCtxGetId): an address is never
 * reused in another context, nor after cudaDeviceReset. Make the first call in each
 * context before any stream capture.
 * All calls on a device share the one array: the part that must start at zero is
 * cleared on the stream at each call, but calls that overlap on the GPU (other streams,
 * other host threads) race on it and must be serialised by the caller.
 */
#define MKV_NOALLOC_SCRATCH_BYTES (16u << 20)
MKV_API int mkv_paged_decode_noalloc(const void* query, int64_t q_stride_seq, int64_t q_stride_head,
                                     int32_t q_dtype, const void* k_cache, const void* v_cache,
                                     int32_t cache_dtype, int64_t num_blocks, int32_t block_size,
                                     const void* block_tables, int32_t block_table_index_type,
                                     int64_t block_table_stride_seq, int32_t max_num_blocks,
                                     const void* context_lens, int32_t context_lens_index_type,
                                     int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                     int32_t head_dim, float scale, void* out,
                                     int64_t out_stride_seq, int64_t out_stride_head,
                                     int32_t num_splits, int32_t* invalid_count, void* stream);

/* ------------------------------------------------------------------------------------
 * Tensor-parallel all-reduce fused with residual add + RMSNorm (decode step, after
 * o_proj and down_proj). Replaces dist.all_reduce in RowParallelLinear.forward
 * (linear.py:222-225) followed by LayerNorm.residual_rms_forward (layernorm.py:25-27):
 *   x = sum over ranks of partial;  s = x + residual;  residual_out <- s;
 *   out = s / sqrt(mean(s^2) + eps) * weight
 * (residual NULL: s = x; residual_out NULL: s is not stored; residual_out may equal
 * residual)
 * with x and s rounded to the data type as the reference's tensor ops round them, sums in
 * fp32 in rank order (every rank computes the same bits).
 * partial: this rank's (num_tokens, hidden) partial, in any device memory. Each rank owns
 * two exchange buffers of at least num_tokens x hidden values, buf_stride bytes apart,
 * and a flag array (MKV_AR_FLAG_BYTES), all in memory the other ranks map with CUDA IPC
 * (mkv_ipc_alloc / mkv_ipc_open, which zero-fill); peer_bufs[r] / peer_flags[r] are rank
 * r's as this process sees them. state: this rank's 8 bytes, zeroed once; the kernel keeps
 * the call count there (call e uses exchange buffer e % 2), so calls need no host-side
 * counter and can be captured in a CUDA graph. Every rank makes the same calls in the
 * same order with the same num_tokens. A wait longer than timeout_cycles (0: about a
 * second) sets *error_flag to 1 and leaves out undefined; no host wait is involved.
 * world_size 1: residual add + RMSNorm of partial (peer arguments and error flag unused).
 * hidden a multiple of 8, at most 8192; bf16 or f16; 16-byte aligned buffers.
 * ---------------------------------------------------------------------------------- */
#define MKV_AR_MAX_RANKS 8
#define MKV_AR_MAX_BLOCKS 128
#define MKV_AR_FLAG_BYTES (MKV_AR_MAX_BLOCKS * MKV_AR_MAX_RANKS * 4)
#define MKV_IPC_HANDLE_BYTES 64

MKV_API int mkv_allreduce_residual_rmsnorm(
    const void* partial, void* const* peer_bufs, int64_t buf_stride, uint32_t* const* peer_flags,
    int32_t rank, int32_t world_size, uint32_t* state, const void* residual, void* residual_out,
    const void* weight, void* out,
    int64_t num_tokens, int32_t hidden, int32_t dtype, float eps, int32_t* error_flag,
    int64_t timeout_cycles, void* stream);

/* Device memory another process can map: cudaMalloc + zero fill + its IPC handle
 * (MKV_IPC_HANDLE_BYTES written to handle_out). */
MKV_API int mkv_ipc_alloc(size_t bytes, void** ptr, void* handle_out);
MKV_API int mkv_ipc_free(void* ptr);
/* Maps another process's mkv_ipc_alloc buffer into this one (peer access enabled). */
MKV_API int mkv_ipc_open(const void* handle, void** ptr);
MKV_API int mkv_ipc_close(void* ptr);

/* ------------------------------------------------------------------------------------
 * Decode-step metadata on the device (replaces the per-step Python loops and three host
 * tensors of ModelRunner.prepare_decode, model_runner.py:631-671). packed (device, int32):
 * [seq_lens (num_seqs)] [block tables (num_seqs x max_blocks), -1 padded], the lengths
 * including the token being decoded. Writes context_lens[b] = seq_lens[b] and
 * slot_mapping[b] = page * block_size + (seq_lens[b] - 1) % block_size for the page
 * holding position seq_lens[b] - 1 (-1 when that page is missing), both int64. The block
 * tables are used in place as the decode's (num_seqs, max_blocks) int32 table.
 * ---------------------------------------------------------------------------------- */
MKV_API int mkv_decode_metadata(const int32_t* packed, int32_t num_seqs, int32_t max_blocks,
                                int32_t block_size, int64_t* slot_mapping, int64_t* context_lens,
                                void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MKV_H_ */
