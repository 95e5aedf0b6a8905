// KV append into block-table pages: same-dtype copy, FP8 E4M3 quantisation with a
// per-tensor scale, the device-side sentinel-aware FP8 scale calibration, and FP8 /
// INT8 quantisation with a dynamic scale per (token, kv head) row.
//
// Reference behaviour (heart1128/mini-kvllm, src/myvllm/layers/attention.py):
//   store_kvcache_kernel       attention.py:7-64    cache.view(-1,KVH,D)[slot] = x, slot -1 skipped
//   store_kvcache_fp8_kernel   attention.py:118-191 e4m3(clamp(x / scale, -448, 448)), per-tensor branch 182-191,
//                                                   per-(token, head) branch 168-181 (scale = amax / 448)
//   store_kvcache_fp8 (host)   attention.py:315-323 scale calibrated once from amax while it is 1.0
//   store_kvcache_int8_kernel  attention.py:195-252 scale = max(amax / 127, 1e-6), round half away
//
// B200 design: the append is pure HBM traffic (one read of the new rows, one write
// into the pages). Each thread moves one 16-byte chunk of a (token, head) row for
// both K and V with a streaming vector load and a vector store; a token's row of
// all heads is contiguous in both the source and the page, so each warp touches
// whole 128-byte lines. The grid is sized in multiples of the SM count.
#include <cstdio>

#include "mkv_common.cuh"

namespace mkv {
namespace {

constexpr int kStoreThreads = 256;

inline int grid_for(int64_t work_items, int threads) {
  int64_t blocks = (work_items + threads - 1) / threads;
  const int64_t cap = (int64_t)kNumSMs * 32;  // enough resident blocks to cover latency
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

// -------------------------------------------------------------------- same-dtype copy
// One thread per 16-byte chunk of a (token, head) row, for K and V.
template <typename SlotT>
__global__ void __launch_bounds__(kStoreThreads)
store_kv_vec16_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                      int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                      uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                      const SlotT* __restrict__ slots, int64_t num_slots, int64_t num_tokens,
                      int num_heads, int row_chunks, int32_t* invalid) {
  const int64_t per_token = (int64_t)num_heads * row_chunks;
  const int64_t total = num_tokens * per_token;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_token;
    const int rem = (int)(i - t * per_token);
    const int h = rem / row_chunks;
    const int c = rem - h * row_chunks;
    const int64_t slot = load_index(slots, t);
    if (slot < 0) continue;  // -1: nothing to store for this token
    if (slot >= num_slots) {
      if (rem == 0 && invalid != nullptr) atomicAdd(invalid, 1);
      continue;
    }
    const uint4 kv = ld_stream_v4(key + t * k_st + h * k_sh + (int64_t)c * 16);
    const uint4 vv = ld_stream_v4(value + t * v_st + h * v_sh + (int64_t)c * 16);
    const int64_t dst = ((slot * num_heads + h) * row_chunks + c) * 16;
    st_v4(k_cache + dst, kv);
    st_v4(v_cache + dst, vv);
  }
}

// Element-wise fallback when rows or strides are not 16-byte aligned.
template <typename T, typename SlotT>
__global__ void __launch_bounds__(kStoreThreads)
store_kv_scalar_kernel(const T* __restrict__ key, const T* __restrict__ value, int64_t k_st,
                       int64_t k_sh, int64_t v_st, int64_t v_sh,  // elements
                       T* __restrict__ k_cache, T* __restrict__ v_cache,
                       const SlotT* __restrict__ slots, int64_t num_slots, int64_t num_tokens,
                       int num_heads, int head_dim, int32_t* invalid) {
  const int64_t per_token = (int64_t)num_heads * head_dim;
  const int64_t total = num_tokens * per_token;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_token;
    const int rem = (int)(i - t * per_token);
    const int h = rem / head_dim;
    const int d = rem - h * head_dim;
    const int64_t slot = load_index(slots, t);
    if (slot < 0) continue;
    if (slot >= num_slots) {
      if (rem == 0 && invalid != nullptr) atomicAdd(invalid, 1);
      continue;
    }
    const int64_t dst = (slot * num_heads + h) * head_dim + d;
    k_cache[dst] = key[t * k_st + h * k_sh + d];
    v_cache[dst] = value[t * v_st + h * v_sh + d];
  }
}

// -------------------------------------------------------------------- FP8 quantise
// clamp(x / scale) with IEEE division, then saturating round-to-nearest-even e4m3.
// fminf/fmaxf return the non-NaN operand, as Triton's tl.minimum/tl.maximum do, so
// a NaN input stores -448 exactly like the reference kernel.
__device__ __forceinline__ uint8_t quantize_e4m3(float x, float scale) {
  float q = x / scale;
  q = fminf(fmaxf(q, -448.0f), 448.0f);
  return f32_to_e4m3(q);
}

template <typename T> struct Vec16 {  // 16 elements of T loaded with 16-byte loads
  static constexpr int kLoads = (16 * (int)sizeof(T)) / 16;
};

template <typename T>
__device__ __forceinline__ void load16(const uint8_t* p, bool vec, float (&x)[16]) {
  if (vec) {
    uint4 raw[Vec16<T>::kLoads];
#pragma unroll
    for (int j = 0; j < Vec16<T>::kLoads; ++j) raw[j] = ld_stream_v4(p + 16 * j);
    const T* e = reinterpret_cast<const T*>(raw);
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = to_f32(e[j]);
  } else {
    const T* e = reinterpret_cast<const T*>(p);
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = to_f32(e[j]);
  }
}

// One thread per 16-element group of a (token, head) row: reads 16 source elements
// of K and of V, writes one 16-byte chunk of e4m3 into each page.
template <typename T, typename SlotT>
__global__ void __launch_bounds__(kStoreThreads)
store_kv_fp8_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                    int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                    uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                    const float* __restrict__ k_scale, const float* __restrict__ v_scale,
                    const SlotT* __restrict__ slots, int64_t num_slots, int64_t num_tokens,
                    int num_heads, int groups_per_row, bool vec, int32_t* invalid) {
  const float ks = __ldg(k_scale);
  const float vs = __ldg(v_scale);
  const int64_t per_token = (int64_t)num_heads * groups_per_row;
  const int64_t total = num_tokens * per_token;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_token;
    const int rem = (int)(i - t * per_token);
    const int h = rem / groups_per_row;
    const int g = rem - h * groups_per_row;
    const int64_t slot = load_index(slots, t);
    if (slot < 0) continue;
    if (slot >= num_slots) {
      if (rem == 0 && invalid != nullptr) atomicAdd(invalid, 1);
      continue;
    }
    const int64_t src_off = (int64_t)g * 16 * (int64_t)sizeof(T);
    float x[16];
    uint32_t packed[4];
    const int64_t dst = ((slot * num_heads + h) * groups_per_row + g) * 16;

    load16<T>(key + t * k_st + h * k_sh + src_off, vec, x);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      packed[w] = (uint32_t)quantize_e4m3(x[4 * w + 0], ks) |
                  ((uint32_t)quantize_e4m3(x[4 * w + 1], ks) << 8) |
                  ((uint32_t)quantize_e4m3(x[4 * w + 2], ks) << 16) |
                  ((uint32_t)quantize_e4m3(x[4 * w + 3], ks) << 24);
    }
    st_v4(k_cache + dst, make_uint4(packed[0], packed[1], packed[2], packed[3]));

    load16<T>(value + t * v_st + h * v_sh + src_off, vec, x);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      packed[w] = (uint32_t)quantize_e4m3(x[4 * w + 0], vs) |
                  ((uint32_t)quantize_e4m3(x[4 * w + 1], vs) << 8) |
                  ((uint32_t)quantize_e4m3(x[4 * w + 2], vs) << 16) |
                  ((uint32_t)quantize_e4m3(x[4 * w + 3], vs) << 24);
    }
    st_v4(v_cache + dst, make_uint4(packed[0], packed[1], packed[2], packed[3]));
  }
}

// -------------------------------------------------------------------- per-(token, head) scales
// clamp(round-half-away(x * (1 / scale)), -128, 127) as int8: the product and the +-0.5
// are separately rounded (no fused multiply-add), as the reference computes them.
__device__ __forceinline__ int8_t quantize_int8(float x, float inv) {
  float q = __fmul_rn(x, inv);
  q = q >= 0.0f ? __fadd_rn(q, 0.5f) : __fadd_rn(q, -0.5f);
  q = fminf(fmaxf(q, -128.0f), 127.0f);
  return (int8_t)__float2int_rz(q);
}

// One group of LPR lanes (a power of two >= head_dim / 16) per (token, kv head) row:
// each lane loads 16 elements of K and of V, the group reduces the row's amax with
// shuffles, and each lane writes its 16 quantised bytes; lane 0 of the group writes
// the row's two scales. The loop is warp-uniform so that every lane takes part in the
// shuffles.
template <typename T, bool kInt8, typename SlotT>
__global__ void __launch_bounds__(kStoreThreads)
store_kv_pth_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                    int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                    uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                    float* __restrict__ k_scales, float* __restrict__ v_scales,
                    const SlotT* __restrict__ slots, int64_t num_slots, int64_t num_tokens,
                    int num_heads, int groups_per_row, int lpr_shift, bool vec,
                    int32_t* invalid) {
  const int lpr = 1 << lpr_shift;
  const int lane = threadIdx.x & 31;
  const int sub = lane & (lpr - 1);
  const int64_t rows = num_tokens * num_heads;
  const int64_t step = ((int64_t)gridDim.x * blockDim.x) >> lpr_shift;
  for (int64_t r0 = ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) >> lpr_shift;
       r0 < rows; r0 += step) {
    const int64_t row = r0 + (lane >> lpr_shift);
    int64_t t = 0, slot = -1;
    int h = 0;
    if (row < rows) {
      t = row / num_heads;
      h = (int)(row - t * num_heads);
      slot = load_index(slots, t);
      if (slot >= num_slots && h == 0 && sub == 0 && invalid != nullptr) atomicAdd(invalid, 1);
    }
    const bool ok = row < rows && slot >= 0 && slot < num_slots;
    const bool has = ok && sub < groups_per_row;
    const int64_t src_off = (int64_t)sub * 16 * (int64_t)sizeof(T);
    const int64_t dst = ((slot * num_heads + h) * groups_per_row + sub) * 16;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const uint8_t* src = which == 0 ? key + t * k_st + h * k_sh : value + t * v_st + h * v_sh;
      float x[16];
      float amax = 0.0f;
      int nan = 0;
      if (has) {
        load16<T>(src + src_off, vec, x);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float a = fabsf(x[j]);
          nan |= isnan(a) ? 1 : 0;
          amax = fmaxf(amax, a);
        }
      }
      for (int o = 1; o < lpr; o <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        nan |= __shfl_xor_sync(0xffffffffu, nan, o);
      }
      float scale;
      if (kInt8) {
        scale = nan ? 1e-6f : fmaxf(amax / 127.0f, 1e-6f);
      } else {
        scale = (!nan && amax > 0.0f) ? amax / 448.0f : 1.0f;
      }
      if (has) {
        uint32_t packed[4];
        if (kInt8) {
          const float inv = 1.0f / scale;
#pragma unroll
          for (int w = 0; w < 4; ++w)
            packed[w] = (uint32_t)(uint8_t)quantize_int8(x[4 * w + 0], inv) |
                        ((uint32_t)(uint8_t)quantize_int8(x[4 * w + 1], inv) << 8) |
                        ((uint32_t)(uint8_t)quantize_int8(x[4 * w + 2], inv) << 16) |
                        ((uint32_t)(uint8_t)quantize_int8(x[4 * w + 3], inv) << 24);
        } else {
#pragma unroll
          for (int w = 0; w < 4; ++w)
            packed[w] = (uint32_t)quantize_e4m3(x[4 * w + 0], scale) |
                        ((uint32_t)quantize_e4m3(x[4 * w + 1], scale) << 8) |
                        ((uint32_t)quantize_e4m3(x[4 * w + 2], scale) << 16) |
                        ((uint32_t)quantize_e4m3(x[4 * w + 3], scale) << 24);
        }
        st_v4((which == 0 ? k_cache : v_cache) + dst,
              make_uint4(packed[0], packed[1], packed[2], packed[3]));
      }
      if (ok && sub == 0) (which == 0 ? k_scales : v_scales)[slot * num_heads + h] = scale;
    }
  }
}

// -------------------------------------------------------------------- FP8 calibration
// The scale torch computes for `x.abs().amax().clamp(min=1e-8) / 448.0` on a CUDA
// tensor of dtype T: clamp's bound is first converted to T, and division by a
// Python (CPU) scalar is a multiplication by the fp32 reciprocal; the result is
// rounded to T, and `.item()` + `fill_` store it exactly in the fp32 scale.
template <typename T> __device__ __forceinline__ float torch_fp8_scale(float amax) {
  const float lower = round_through<T>(1e-8f);
  const float a = isnan(amax) ? amax : fmaxf(amax, lower);
  const float inv448 = 1.0f / 448.0f;
  return round_through<T>(a * inv448);
}

struct CalibWork {  // MKV_FP8_CALIB_WORK_BYTES bytes, zero between calls
  unsigned int amax_bits[2];
  unsigned int arrived[2];
};
static_assert(sizeof(CalibWork) == MKV_FP8_CALIB_WORK_BYTES, "calibration work layout");

// blockIdx.y selects K (0) or V (1). Every block first checks the sentinel; when the
// scale is already calibrated all blocks return at once (the steady state: one
// 4-byte read). Otherwise each block reduces |x| over a grid-stride range, folds it
// into amax_bits with atomicMax on the IEEE bits (|x| >= 0 orders like unsigned and
// NaN sorts above +inf, so NaN propagates as in torch.amax), and the last block to
// arrive writes the scale and zeroes the work words for the next call.
template <typename T>
__global__ void __launch_bounds__(kStoreThreads)
fp8_calibrate_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                     int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                     int64_t num_tokens, int num_heads, int head_dim, bool vec,
                     float* __restrict__ k_scale, float* __restrict__ v_scale, CalibWork* work) {
  const int which = blockIdx.y;
  float* scale = which ? v_scale : k_scale;
  if (*((volatile float*)scale) != 1.0f) return;  // already calibrated: frozen
  const uint8_t* src = which ? value : key;
  const int64_t st = which ? v_st : k_st;
  const int64_t sh = which ? v_sh : k_sh;

  float m = 0.0f;
  if (vec) {  // rows of head_dim*sizeof(T) bytes in 16-byte chunks
    constexpr int kPer = 16 / (int)sizeof(T);
    const int chunks = head_dim / kPer;
    const int64_t per_token = (int64_t)num_heads * chunks;
    const int64_t total = num_tokens * per_token;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t t = i / per_token;
      const int rem = (int)(i - t * per_token);
      const int h = rem / chunks;
      const int c = rem - h * chunks;
      const uint4 raw = ld_stream_v4(src + t * st + h * sh + (int64_t)c * 16);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const float a = fabsf(to_f32(e[j]));
        m = (a > m || isnan(a)) ? a : m;
      }
    }
  } else {
    const int64_t per_token = (int64_t)num_heads * head_dim;
    const int64_t total = num_tokens * per_token;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t t = i / per_token;
      const int rem = (int)(i - t * per_token);
      const int h = rem / head_dim;
      const int d = rem - h * head_dim;
      const float a = fabsf(to_f32(*reinterpret_cast<const T*>(src + t * st + h * sh +
                                                                  (int64_t)d * sizeof(T))));
      m = (a > m || isnan(a)) ? a : m;
    }
  }
  // Block reduction on the bit patterns (non-negative floats order as unsigned).
  unsigned int bits = __float_as_uint(m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
  __shared__ unsigned int warp_bits[kStoreThreads / 32];
  __shared__ bool is_last;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) warp_bits[wid] = bits;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int b = 0;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) b = max(b, warp_bits[w]);
    atomicMax(&work->amax_bits[which], b);
    __threadfence();
    const unsigned int prev = atomicAdd(&work->arrived[which], 1u);
    is_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (is_last && threadIdx.x == 0) {
    __threadfence();
    const unsigned int b = atomicExch(&work->amax_bits[which], 0u);
    atomicExch(&work->arrived[which], 0u);
    *scale = torch_fp8_scale<T>(__uint_as_float(b));
  }
}

// -------------------------------------------------------------------- host helpers
int check_common(const void* key, const void* value, void* k_cache, void* v_cache,
                 const void* slots, int slot_type, int64_t num_blocks, int block_size,
                 int64_t num_tokens, int num_kv_heads, int head_dim, const char* fn) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks < 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "%s: bad sizes (num_tokens=%lld, num_kv_heads=%d, head_dim=%d, "
                     "block_size=%d, num_blocks=%lld)",
                     fn, (long long)num_tokens, num_kv_heads, head_dim, block_size,
                     (long long)num_blocks);
  if (num_tokens > 0 && (!key || !value || !k_cache || !v_cache || !slots))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (slot_type != MKV_INDEX_I32 && slot_type != MKV_INDEX_I64)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: slot_index_type must be MKV_INDEX_I32 or I64",
                     fn);
  return MKV_OK;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

template <typename T, typename SlotT>
int launch_store(const void* key, const void* value, int64_t k_st, int64_t k_sh, int64_t v_st,
                 int64_t v_sh, void* k_cache, void* v_cache, int64_t num_slots,
                 const SlotT* slots, int64_t num_tokens, int num_heads, int head_dim,
                 int32_t* invalid, cudaStream_t stream) {
  const int64_t eb = sizeof(T);
  const int64_t row_bytes = head_dim * eb;
  const bool vec = (row_bytes % 16 == 0) && aligned16(key) && aligned16(value) &&
                   aligned16(k_cache) && aligned16(v_cache) && ((k_st * eb) % 16 == 0) &&
                   ((k_sh * eb) % 16 == 0) && ((v_st * eb) % 16 == 0) &&
                   ((v_sh * eb) % 16 == 0);
  if (vec) {
    const int row_chunks = (int)(row_bytes / 16);
    const int grid = grid_for(num_tokens * num_heads * row_chunks, kStoreThreads);
    store_kv_vec16_kernel<SlotT><<<grid, kStoreThreads, 0, stream>>>(
        (const uint8_t*)key, (const uint8_t*)value, k_st * eb, k_sh * eb, v_st * eb, v_sh * eb,
        (uint8_t*)k_cache, (uint8_t*)v_cache, slots, num_slots, num_tokens, num_heads,
        row_chunks, invalid);
  } else {
    const int grid = grid_for(num_tokens * num_heads * head_dim, kStoreThreads);
    store_kv_scalar_kernel<T, SlotT><<<grid, kStoreThreads, 0, stream>>>(
        (const T*)key, (const T*)value, k_st, k_sh, v_st, v_sh, (T*)k_cache, (T*)v_cache, slots,
        num_slots, num_tokens, num_heads, head_dim, invalid);
  }
  return cuda_status(cudaGetLastError(), "store_kvcache launch");
}

template <typename T, typename SlotT>
int launch_store_fp8(const void* key, const void* value, int64_t k_st, int64_t k_sh,
                     int64_t v_st, int64_t v_sh, void* k_cache, void* v_cache,
                     const float* k_scale, const float* v_scale, int64_t num_slots,
                     const SlotT* slots, int64_t num_tokens, int num_heads, int head_dim,
                     int32_t* invalid, cudaStream_t stream) {
  const int64_t eb = sizeof(T);
  const bool vec = aligned16(key) && aligned16(value) && ((k_st * eb) % 16 == 0) &&
                   ((k_sh * eb) % 16 == 0) && ((v_st * eb) % 16 == 0) &&
                   ((v_sh * eb) % 16 == 0);
  const int groups = head_dim / 16;
  const int grid = grid_for(num_tokens * num_heads * groups, kStoreThreads);
  store_kv_fp8_kernel<T, SlotT><<<grid, kStoreThreads, 0, stream>>>(
      (const uint8_t*)key, (const uint8_t*)value, k_st * eb, k_sh * eb, v_st * eb, v_sh * eb,
      (uint8_t*)k_cache, (uint8_t*)v_cache, k_scale, v_scale, slots, num_slots, num_tokens,
      num_heads, groups, vec, invalid);
  return cuda_status(cudaGetLastError(), "store_kvcache_fp8 launch");
}

template <typename T, bool kInt8, typename SlotT>
int launch_store_pth(const void* key, const void* value, int64_t k_st, int64_t k_sh,
                     int64_t v_st, int64_t v_sh, void* k_cache, void* v_cache, float* k_scales,
                     float* v_scales, int64_t num_slots, const SlotT* slots, int64_t num_tokens,
                     int num_heads, int head_dim, int32_t* invalid, cudaStream_t stream) {
  const int64_t eb = sizeof(T);
  const bool vec = aligned16(key) && aligned16(value) && ((k_st * eb) % 16 == 0) &&
                   ((k_sh * eb) % 16 == 0) && ((v_st * eb) % 16 == 0) &&
                   ((v_sh * eb) % 16 == 0);
  const int groups = head_dim / 16;
  int lpr_shift = 0;
  while ((1 << lpr_shift) < groups) ++lpr_shift;
  const int grid = grid_for(num_tokens * num_heads << lpr_shift, kStoreThreads);
  store_kv_pth_kernel<T, kInt8, SlotT><<<grid, kStoreThreads, 0, stream>>>(
      (const uint8_t*)key, (const uint8_t*)value, k_st * eb, k_sh * eb, v_st * eb, v_sh * eb,
      (uint8_t*)k_cache, (uint8_t*)v_cache, k_scales, v_scales, slots, num_slots, num_tokens,
      num_heads, groups, lpr_shift, vec, invalid);
  return cuda_status(cudaGetLastError(), "store_kvcache_quant_per_token_head launch");
}

template <typename T>
int launch_calibrate(const void* key, const void* value, int64_t k_st, int64_t k_sh,
                     int64_t v_st, int64_t v_sh, int64_t num_tokens, int num_heads, int head_dim,
                     float* k_scale, float* v_scale, void* work, cudaStream_t stream) {
  const int64_t eb = sizeof(T);
  const bool vec = ((head_dim * eb) % 16 == 0) && aligned16(key) && aligned16(value) &&
                   ((k_st * eb) % 16 == 0) && ((k_sh * eb) % 16 == 0) &&
                   ((v_st * eb) % 16 == 0) && ((v_sh * eb) % 16 == 0);
  const int64_t items = vec ? num_tokens * num_heads * (head_dim * eb / 16)
                            : num_tokens * num_heads * head_dim;
  int blocks = grid_for(items, kStoreThreads);
  if (blocks > kNumSMs * 4) blocks = kNumSMs * 4;  // the reduction needs few blocks
  dim3 grid(blocks, 2);
  fp8_calibrate_kernel<T><<<grid, kStoreThreads, 0, stream>>>(
      (const uint8_t*)key, (const uint8_t*)value, k_st * eb, k_sh * eb, v_st * eb, v_sh * eb,
      num_tokens, num_heads, head_dim, vec, k_scale, v_scale, (CalibWork*)work);
  return cuda_status(cudaGetLastError(), "calibrate_fp8_scales launch");
}

}  // namespace
}  // namespace mkv

using namespace mkv;

extern "C" int mkv_store_kvcache(const void* key, const void* value, int64_t key_stride_token,
                                 int64_t key_stride_head, int64_t value_stride_token,
                                 int64_t value_stride_head, void* k_cache, void* v_cache,
                                 int64_t num_blocks, int32_t block_size, const void* slot_mapping,
                                 int32_t slot_index_type, int64_t num_tokens,
                                 int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                                 int32_t* invalid_count, void* stream) {
  clear_error();
  int st = check_common(key, value, k_cache, v_cache, slot_mapping, slot_index_type, num_blocks,
                        block_size, num_tokens, num_kv_heads, head_dim, "mkv_store_kvcache");
  if (st != MKV_OK) return st;
  if (num_tokens == 0) return MKV_OK;
  const int64_t num_slots = num_blocks * block_size;
  cudaStream_t s = (cudaStream_t)stream;
  const bool i64 = slot_index_type == MKV_INDEX_I64;
#define MKV_STORE(T)                                                                          \
  return i64 ? launch_store<T, int64_t>(key, value, key_stride_token, key_stride_head,        \
                                        value_stride_token, value_stride_head, k_cache,       \
                                        v_cache, num_slots, (const int64_t*)slot_mapping,     \
                                        num_tokens, num_kv_heads, head_dim, invalid_count, s) \
             : launch_store<T, int32_t>(key, value, key_stride_token, key_stride_head,        \
                                        value_stride_token, value_stride_head, k_cache,       \
                                        v_cache, num_slots, (const int32_t*)slot_mapping,     \
                                        num_tokens, num_kv_heads, head_dim, invalid_count, s)
  switch (dtype) {
    case MKV_DTYPE_F32: MKV_STORE(float);
    case MKV_DTYPE_F16: MKV_STORE(f16);
    case MKV_DTYPE_BF16: MKV_STORE(bf16);
    case MKV_DTYPE_FP8_E4M3: MKV_STORE(uint8_t);
    default:
      return set_error(MKV_ERR_UNSUPPORTED, "mkv_store_kvcache: unsupported dtype %d", dtype);
  }
#undef MKV_STORE
}

extern "C" int mkv_calibrate_fp8_scales(const void* key, const void* value,
                                        int64_t key_stride_token, int64_t key_stride_head,
                                        int64_t value_stride_token, int64_t value_stride_head,
                                        int64_t num_tokens, int32_t num_kv_heads,
                                        int32_t head_dim, int32_t dtype, float* k_scale,
                                        float* v_scale, void* work, void* stream) {
  clear_error();
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "mkv_calibrate_fp8_scales: bad sizes");
  if (!k_scale || !v_scale || !work || (num_tokens > 0 && (!key || !value)))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "mkv_calibrate_fp8_scales: null pointer argument");
  if (((uintptr_t)work & 7u) != 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "mkv_calibrate_fp8_scales: work must be 8-byte aligned");
  if (num_tokens == 0) return MKV_OK;  // no data: the scales stay as they are
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case MKV_DTYPE_F32:
      return launch_calibrate<float>(key, value, key_stride_token, key_stride_head,
                                     value_stride_token, value_stride_head, num_tokens,
                                     num_kv_heads, head_dim, k_scale, v_scale, work, s);
    case MKV_DTYPE_F16:
      return launch_calibrate<f16>(key, value, key_stride_token, key_stride_head,
                                   value_stride_token, value_stride_head, num_tokens,
                                   num_kv_heads, head_dim, k_scale, v_scale, work, s);
    case MKV_DTYPE_BF16:
      return launch_calibrate<bf16>(key, value, key_stride_token, key_stride_head,
                                    value_stride_token, value_stride_head, num_tokens,
                                    num_kv_heads, head_dim, k_scale, v_scale, work, s);
    default:
      return set_error(MKV_ERR_UNSUPPORTED,
                       "mkv_calibrate_fp8_scales: key dtype must be f32, f16 or bf16 (got %d)",
                       dtype);
  }
}

extern "C" int mkv_store_kvcache_fp8(const void* key, const void* value,
                                     int64_t key_stride_token, int64_t key_stride_head,
                                     int64_t value_stride_token, int64_t value_stride_head,
                                     void* k_cache, void* v_cache, const float* k_scale,
                                     const float* v_scale, int64_t num_blocks,
                                     int32_t block_size, const void* slot_mapping,
                                     int32_t slot_index_type, int64_t num_tokens,
                                     int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                                     int32_t* invalid_count, void* stream) {
  clear_error();
  int st = check_common(key, value, k_cache, v_cache, slot_mapping, slot_index_type, num_blocks,
                        block_size, num_tokens, num_kv_heads, head_dim, "mkv_store_kvcache_fp8");
  if (st != MKV_OK) return st;
  if (head_dim % 16 != 0)
    return set_error(MKV_ERR_UNSUPPORTED,
                     "mkv_store_kvcache_fp8: head_dim must be a multiple of 16 (got %d)",
                     head_dim);
  if (!k_scale || !v_scale)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "mkv_store_kvcache_fp8: null scale pointer");
  if ((((uintptr_t)k_cache) & 15u) || (((uintptr_t)v_cache) & 15u))
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "mkv_store_kvcache_fp8: caches must be 16-byte aligned");
  if (num_tokens == 0) return MKV_OK;
  const int64_t num_slots = num_blocks * block_size;
  cudaStream_t s = (cudaStream_t)stream;
  const bool i64 = slot_index_type == MKV_INDEX_I64;
#define MKV_STORE8(T)                                                                          \
  return i64 ? launch_store_fp8<T, int64_t>(key, value, key_stride_token, key_stride_head,     \
                                            value_stride_token, value_stride_head, k_cache,    \
                                            v_cache, k_scale, v_scale, num_slots,              \
                                            (const int64_t*)slot_mapping, num_tokens,          \
                                            num_kv_heads, head_dim, invalid_count, s)          \
             : launch_store_fp8<T, int32_t>(key, value, key_stride_token, key_stride_head,     \
                                            value_stride_token, value_stride_head, k_cache,    \
                                            v_cache, k_scale, v_scale, num_slots,              \
                                            (const int32_t*)slot_mapping, num_tokens,          \
                                            num_kv_heads, head_dim, invalid_count, s)
  switch (dtype) {
    case MKV_DTYPE_F32: MKV_STORE8(float);
    case MKV_DTYPE_F16: MKV_STORE8(f16);
    case MKV_DTYPE_BF16: MKV_STORE8(bf16);
    default:
      return set_error(MKV_ERR_UNSUPPORTED,
                       "mkv_store_kvcache_fp8: key dtype must be f32, f16 or bf16 (got %d)", dtype);
  }
#undef MKV_STORE8
}

extern "C" int mkv_store_kvcache_quant_per_token_head(
    const void* key, const void* value, int64_t key_stride_token, int64_t key_stride_head,
    int64_t value_stride_token, int64_t value_stride_head, void* k_cache, void* v_cache,
    int32_t cache_dtype, float* k_scales, float* v_scales, int64_t num_blocks,
    int32_t block_size, const void* slot_mapping, int32_t slot_index_type, int64_t num_tokens,
    int32_t num_kv_heads, int32_t head_dim, int32_t dtype, int32_t* invalid_count, void* stream) {
  clear_error();
  const char* fn = "mkv_store_kvcache_quant_per_token_head";
  int st = check_common(key, value, k_cache, v_cache, slot_mapping, slot_index_type, num_blocks,
                        block_size, num_tokens, num_kv_heads, head_dim, fn);
  if (st != MKV_OK) return st;
  if (cache_dtype != MKV_DTYPE_FP8_E4M3 && cache_dtype != MKV_DTYPE_INT8)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: cache_dtype must be FP8_E4M3 or INT8 (got %d)", fn,
                     cache_dtype);
  if (head_dim % 16 != 0 || head_dim > 512)
    return set_error(MKV_ERR_UNSUPPORTED,
                     "%s: head_dim must be a multiple of 16 and at most 512 (got %d)", fn,
                     head_dim);
  if (!k_scales || !v_scales)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: null scale pointer", fn);
  if ((((uintptr_t)k_scales) & 3u) || (((uintptr_t)v_scales) & 3u))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: scales must be 4-byte aligned", fn);
  if ((((uintptr_t)k_cache) & 15u) || (((uintptr_t)v_cache) & 15u))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: caches must be 16-byte aligned", fn);
  if (num_tokens == 0) return MKV_OK;
  const int64_t num_slots = num_blocks * block_size;
  cudaStream_t s = (cudaStream_t)stream;
  const bool i64 = slot_index_type == MKV_INDEX_I64;
  const bool i8 = cache_dtype == MKV_DTYPE_INT8;
#define MKV_PTH(T, I8)                                                                          \
  return i64 ? launch_store_pth<T, I8, int64_t>(key, value, key_stride_token, key_stride_head,  \
                                                value_stride_token, value_stride_head, k_cache, \
                                                v_cache, k_scales, v_scales, num_slots,         \
                                                (const int64_t*)slot_mapping, num_tokens,       \
                                                num_kv_heads, head_dim, invalid_count, s)       \
             : launch_store_pth<T, I8, int32_t>(key, value, key_stride_token, key_stride_head,  \
                                                value_stride_token, value_stride_head, k_cache, \
                                                v_cache, k_scales, v_scales, num_slots,         \
                                                (const int32_t*)slot_mapping, num_tokens,       \
                                                num_kv_heads, head_dim, invalid_count, s)
  switch (dtype) {
    case MKV_DTYPE_F32:
      if (i8) MKV_PTH(float, true);
      MKV_PTH(float, false);
    case MKV_DTYPE_F16:
      if (i8) MKV_PTH(f16, true);
      MKV_PTH(f16, false);
    case MKV_DTYPE_BF16:
      if (i8) MKV_PTH(bf16, true);
      MKV_PTH(bf16, false);
    default:
      return set_error(MKV_ERR_UNSUPPORTED, "%s: key dtype must be f32, f16 or bf16 (got %d)", fn,
                       dtype);
  }
#undef MKV_PTH
}

// ============================================================ decode-step metadata
// Per-step decode metadata of ModelRunner.prepare_decode (model_runner.py:631-671) from a
// packed table kept on the device: packed = [seq_lens (B)] [block tables (B x W), -1
// padded], int32. Sequence b decodes its token at position seq_lens[b] - 1:
//   context_lens[b] = seq_lens[b]; slot_mapping[b] = page * block_size + offset of that
//   position (the reference's block_table[-1] * block_size + last_block_num_tokens - 1),
//   -1 when the page is missing (the append then skips the token).
namespace mkv {
namespace {
__global__ void decode_metadata_kernel(const int32_t* packed, int B, int W, int block_size,
                                       int64_t* slot_mapping, int64_t* context_lens) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int n = packed[b];
  context_lens[b] = n;
  int64_t slot = -1;
  if (n > 0) {
    const int blk = (n - 1) / block_size;
    const int page = blk < W ? packed[B + (int64_t)b * W + blk] : -1;
    if (page >= 0) slot = (int64_t)page * block_size + (n - 1) % block_size;
  }
  slot_mapping[b] = slot;
}
}  // namespace
}  // namespace mkv

extern "C" int mkv_decode_metadata(const int32_t* packed, int32_t num_seqs, int32_t max_blocks,
                                   int32_t block_size, int64_t* slot_mapping, int64_t* context_lens,
                                   void* stream) {
  clear_error();
  if (num_seqs < 0 || max_blocks < 0 || block_size <= 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "mkv_decode_metadata: bad sizes");
  if (num_seqs == 0) return MKV_OK;
  if (!packed || !slot_mapping || !context_lens)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "mkv_decode_metadata: null pointer argument");
  mkv::decode_metadata_kernel<<<(num_seqs + 127) / 128, 128, 0, (cudaStream_t)stream>>>(
      packed, num_seqs, max_blocks, block_size, slot_mapping, context_lens);
  return cuda_status(cudaGetLastError(), "decode_metadata launch");
}
