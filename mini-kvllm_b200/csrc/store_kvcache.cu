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
// into the pages) over a few MB, so it is bound by how many bytes are in flight and by
// the launch itself. Each thread owns CHUNKS 16-byte chunks of K and of V (or 16-element
// groups for the quantisers), issues every load of them before its first store, and
// the chunk index advances by the grid's thread count, so each warp instruction touches
// whole 128-byte lines. One wave of CTAs then holds the whole batch in flight. A
// token's row of all heads is contiguous in both the source and the page.
// The FP8 per-tensor store reads the scale itself and calibrates it in the same launch
// while it still holds the 1.0 sentinel (the last CTA to finish the amax reduction
// quantises the batch), so a calibrated step is one launch.
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

// Items per thread: as many as keep at least two CTAs of work per SM, up to 4 (one wave
// then holds a config-2 batch of 4096 tokens entirely in flight); small batches (a
// decode step's few hundred tokens) spread one item per thread over more SMs.
inline int per_thread_items(int64_t items) {
  const int64_t min_threads = (int64_t)kNumSMs * 2 * kStoreThreads;
  if (items >= 4 * min_threads) return 4;
  if (items >= 2 * min_threads) return 2;
  return 1;
}

// Blocks rounded up to a multiple of the SM count, so that every SM gets the same
// number of CTAs (the kernels' loops leave surplus threads idle).
inline int sm_multiple(int blocks) { return (blocks + kNumSMs - 1) / kNumSMs * kNumSMs; }

inline int log2_if_pow2(int64_t x) {
  if (x <= 0 || (x & (x - 1)) != 0) return -1;
  int s = 0;
  while (((int64_t)1 << s) < x) ++s;
  return s;
}

// -------------------------------------------------------------------- same-dtype copy
// CHUNKS 16-byte chunks of K and of V per thread, strided by the grid's thread count:
// all 2 * CHUNKS loads (and the slot loads) are in flight before the first store.
// Indices are 32-bit (the host takes this kernel only below 2^31 chunks).
template <typename SlotT, int CHUNKS>
__global__ void __launch_bounds__(kStoreThreads)
store_kv_copy_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                     int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                     uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                     const SlotT* __restrict__ slots, int64_t num_slots, uint32_t total,
                     uint32_t num_heads, uint32_t row_chunks, int pt_shift, int rc_shift,
                     int32_t* invalid) {
  pdl_trigger();  // a dependent decode may begin its prologue now
  const uint32_t per_token = num_heads * row_chunks;
  const uint32_t nthreads = gridDim.x * blockDim.x;
  for (uint32_t base = blockIdx.x * blockDim.x + threadIdx.x; base < total;
       base += nthreads * CHUNKS) {
    uint4 kv[CHUNKS], vv[CHUNKS];
    int64_t dst[CHUNKS];
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
      const uint32_t i = base + (uint32_t)j * nthreads;
      dst[j] = -1;
      if (i < total) {
        // shifts when the sizes are powers of two (pt_shift / rc_shift >= 0)
        const uint32_t t = pt_shift >= 0 ? i >> pt_shift : i / per_token;
        const uint32_t rem = i - t * per_token;
        const uint32_t h = rc_shift >= 0 ? rem >> rc_shift : rem / row_chunks;
        const uint32_t c = rem - h * row_chunks;
        const int64_t slot = load_index(slots, (int64_t)t);
        kv[j] = ld_stream_v4(key + (int64_t)t * k_st + (int64_t)h * k_sh + c * 16u);
        vv[j] = ld_stream_v4(value + (int64_t)t * v_st + (int64_t)h * v_sh + c * 16u);
        if (slot >= 0 && slot < num_slots) {
          dst[j] = ((slot * num_heads + h) * row_chunks + c) * 16;
        } else if (slot >= num_slots && rem == 0 && invalid != nullptr) {
          atomicAdd(invalid, 1);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
      if (dst[j] >= 0) {
        st_v4(k_cache + dst[j], kv[j]);
        st_v4(v_cache + dst[j], vv[j]);
      }
    }
  }
}

// One thread per 16-byte chunk of a (token, head) row, for K and V (beyond 2^31 chunks).
template <typename SlotT>
__global__ void __launch_bounds__(kStoreThreads)
store_kv_vec16_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                      int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                      uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                      const SlotT* __restrict__ slots, int64_t num_slots, int64_t num_tokens,
                      int num_heads, int row_chunks, int32_t* invalid) {
  pdl_trigger();  // a dependent decode may begin its prologue now
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
  pdl_trigger();  // a dependent decode may begin its prologue now
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
  pdl_trigger();  // a dependent decode may begin its prologue now
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

// Two quotients as e4m3 bytes, element `lo` in the low byte: one round-to-nearest-even
// conversion for the pair that saturates finite values beyond +-448 and infinities to
// +-448 (NaN would stay NaN; the callers never pass one).
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return (uint32_t)r;
}

// Division by one scale, correctly rounded like IEEE x / scale, in one multiply and two
// FMAs (Markstein's method), two quotients at a time with the packed fp32 instructions:
// y = RN(1 / scale) is taken once by IEEE division; q = RN(x * y) is then within about
// an ulp of x / scale, the remainder r = x - q * scale is exact in an FMA, and
// RN(q + r * y) is the correctly rounded quotient. Only quotients within the e4m3 range
// matter (the conversion saturates everything beyond +-448), so q is capped at 464 before
// the correction and the result is floored at -464 after it; then no case needs a branch:
//   +inf or a positive overflow -> a large or infinite quotient -> saturates to 448;
//   -inf or a negative overflow -> NaN from inf - inf or a large negative quotient -> -464
//   (NaN is floored to -464, as fmaxf keeps the number) -> -448;
//   NaN x -> NaN -> -464 -> -448, the reference's clamp(NaN) (fmax/fmin keep the number);
// and copysign restores the sign of an exact zero quotient. A scale that is not a
// normal number, or whose reciprocal is not, takes the IEEE division itself (one uniform
// branch per 16 elements). Tests compare the bytes with IEEE division at every e4m3
// rounding midpoint for many scales.
struct ScaleDiv {
  float s, y;
  uint64_t y2, ns2;  // (y, y) and (-s, -s) for the packed instructions
  bool fast;
  __device__ __forceinline__ explicit ScaleDiv(float scale) : s(scale) {
    y = 1.0f / scale;
    const float as = fabsf(scale), ay = fabsf(y);
    fast = as >= 0x1p-126f && as <= 0x1p126f && ay >= 0x1p-126f && ay <= 0x1p126f;
    y2 = f2_pack(y, y);
    ns2 = f2_pack(-scale, -scale);
  }
  // two quotients ready for the saturating e4m3 conversion (fast path)
  __device__ __forceinline__ void quot2(float x0, float x1, float& c0, float& c1) const {
    const uint64_t x2 = f2_pack(x0, x1);
    float q0, q1;
    f2_unpack(f2_mul(x2, y2), q0, q1);
    const uint64_t a2 = f2_pack(fminf(q0, 464.0f), fminf(q1, 464.0f));
    const uint64_t r2 = f2_fma(a2, ns2, x2);  // x - a * scale, exact
    float b0, b1;
    f2_unpack(f2_fma(r2, y2, a2), b0, b1);
    c0 = fmaxf(copysignf(b0, q0), -464.0f);
    c1 = fmaxf(copysignf(b1, q1), -464.0f);
  }
  // the same from IEEE division (scales that are not normal numbers)
  __device__ __forceinline__ void quot2_ieee(float x0, float x1, float& c0, float& c1) const {
    c0 = fminf(fmaxf(x0 / s, -448.0f), 448.0f);
    c1 = fminf(fmaxf(x1 / s, -448.0f), 448.0f);
  }
};

// Four quantised elements (a..d, a lowest) as e4m3 bytes with the saturating conversion.
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  return e4m3x2(a, b) | (e4m3x2(c, d) << 16);
}

// 16 elements quantised with one scale, packed as 16 e4m3 bytes (element 0 lowest).
template <typename Get>
__device__ __forceinline__ uint4 quantize16_from(const Get& at, const ScaleDiv& d) {
  uint32_t w[4];
  if (d.fast) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float c0, c1, c2, c3;
      d.quot2(at(4 * i), at(4 * i + 1), c0, c1);
      d.quot2(at(4 * i + 2), at(4 * i + 3), c2, c3);
      w[i] = e4m3x4(c0, c1, c2, c3);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float c0, c1, c2, c3;
      d.quot2_ieee(at(4 * i), at(4 * i + 1), c0, c1);
      d.quot2_ieee(at(4 * i + 2), at(4 * i + 3), c2, c3);
      w[i] = e4m3x4(c0, c1, c2, c3);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ uint4 quantize16(const float (&x)[16], const ScaleDiv& d) {
  return quantize16_from([&](int j) { return x[j]; }, d);
}

// The 16-element group of a (token, head) row as raw 16-byte words, converted to float
// only after every load of the thread is in flight.
template <typename T> struct Raw16 {
  static constexpr int kWords = 16 * (int)sizeof(T) / 16;
  uint4 w[kWords];
  __device__ __forceinline__ void load(const uint8_t* p) {
#pragma unroll
    for (int j = 0; j < kWords; ++j) w[j] = ld_stream_v4(p + 16 * j);
  }
  __device__ __forceinline__ float at(int j) const { return to_f32(reinterpret_cast<const T*>(w)[j]); }
  __device__ __forceinline__ void get(float (&x)[16]) const {
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = at(j);
  }
  // the 16 elements quantised with one scale as 16 e4m3 bytes, converted pair by pair
  __device__ __forceinline__ uint4 quantize(const ScaleDiv& d) const {
    return quantize16_from([&](int j) { return at(j); }, d);
  }
};

__device__ __forceinline__ float amax_step(float m, float a) {  // NaN wins, as torch.amax
  return (a > m || isnan(a)) ? a : m;
}

// FP8 per-tensor append in one launch, calibrating a scale that still holds the 1.0
// sentinel (attention.py:315-323) before quantising with it (118-191). Each thread owns
// GROUPS 16-element groups of K and of V, strided by the grid's thread count; their
// loads and the two scale loads are all issued before anything is computed.
//   Steady state (both scales calibrated, or work == nullptr): quantise and store.
//   Calibration (a sentinel seen; every CTA reads the scales before any CTA can write
//   them, so all agree): each CTA folds |x| of its share of the batch into
//   work->amax_bits with atomicMax on the IEEE bits and stores nothing; the last CTA to
//   arrive writes the scale(s), leaves the work words at zero, and quantises and stores
//   the whole batch itself. No CTA waits for another, so the launch can neither hang nor
//   depend on how many CTAs are resident; the single-CTA store is paid once per layer.
// The vector form needs 16-byte aligned rows and strides (kVec); otherwise GROUPS = 1
// and elements are loaded one by one.
template <typename T, typename SlotT, int GROUPS, bool kVec>
__global__ void __launch_bounds__(kStoreThreads, 4)
store_kv_fp8_calib_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                          int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                          uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                          float* k_scale, float* v_scale, const SlotT* __restrict__ slots,
                          int64_t num_slots, uint32_t total, uint32_t num_heads,
                          uint32_t groups_per_row, int pt_shift, int gr_shift, CalibWork* work,
                          int32_t* invalid) {
  pdl_trigger();  // a dependent decode may begin its prologue now
  const uint32_t per_token = num_heads * groups_per_row;
  const uint32_t nthreads = gridDim.x * blockDim.x;
  const uint32_t tid0 = blockIdx.x * blockDim.x + threadIdx.x;
  constexpr int64_t kGroupBytes = 16 * (int64_t)sizeof(T);

  struct Item {
    int64_t slot;
    uint32_t t, h, g;
  };
  auto locate = [&](uint32_t i, Item& it) {  // shifts when the sizes are powers of two
    it.t = pt_shift >= 0 ? i >> pt_shift : i / per_token;
    const uint32_t rem = i - it.t * per_token;
    it.h = gr_shift >= 0 ? rem >> gr_shift : rem / groups_per_row;
    it.g = rem - it.h * groups_per_row;
    it.slot = load_index(slots, (int64_t)it.t);
  };
  auto src_k = [&](const Item& it) { return key + (int64_t)it.t * k_st + (int64_t)it.h * k_sh + it.g * kGroupBytes; };
  auto src_v = [&](const Item& it) { return value + (int64_t)it.t * v_st + (int64_t)it.h * v_sh + it.g * kGroupBytes; };
  auto load_vals = [&](const uint8_t* p, float (&x)[16]) {  // scalar form (kVec false)
    const T* e = reinterpret_cast<const T*>(p);
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = to_f32(e[j]);
  };
  // quantise + store one group whose values are in xk / xv
  auto store_group = [&](const Item& it, const float (&xk)[16], const float (&xv)[16],
                         const ScaleDiv& ks, const ScaleDiv& vs, bool count_invalid) {
    if (it.slot < 0) return;  // -1: nothing to store for this token
    if (it.slot >= num_slots) {
      if (count_invalid && it.h == 0 && it.g == 0 && invalid != nullptr) atomicAdd(invalid, 1);
      return;
    }
    const int64_t dst = ((it.slot * num_heads + it.h) * groups_per_row + it.g) * 16;
    st_v4(k_cache + dst, quantize16(xk, ks));
    st_v4(v_cache + dst, quantize16(xv, vs));
  };

  // Destination of a group: -1 nothing to store (slot -1), -2 out-of-range slot (counted
  // once per token when the group is stored, never while only loaded).
  auto dest = [&](const Item& it) -> int64_t {
    if (it.slot < 0) return -1;
    if (it.slot >= num_slots) return (it.h == 0 && it.g == 0) ? -2 : -1;
    return ((it.slot * num_heads + it.h) * groups_per_row + it.g) * 16;
  };

  // ---- first stride of groups: loads, then the scales, all in flight together
  int64_t dst[GROUPS];
  uint32_t base = tid0;
  Raw16<T> rk[kVec ? GROUPS : 1], rv[kVec ? GROUPS : 1];
  Item it1;  // the scalar form's group (GROUPS == 1)
  auto load_stride = [&]() {
#pragma unroll
    for (int j = 0; j < GROUPS; ++j) {
      const uint32_t i = base + (uint32_t)j * nthreads;
      dst[j] = -1;
      if (i < total) {
        Item it;
        locate(i, it);
        if constexpr (kVec) {
          rk[j].load(src_k(it));
          rv[j].load(src_v(it));
        } else {
          it1 = it;
        }
        dst[j] = dest(it);
      }
    }
  };
  load_stride();
  const float ks = *reinterpret_cast<volatile const float*>(k_scale);
  const float vs = *reinterpret_cast<volatile const float*>(v_scale);
  const bool need_k = work != nullptr && ks == 1.0f;
  const bool need_v = work != nullptr && vs == 1.0f;

  if (!need_k && !need_v) {  // ------------------------------------ steady state
    const ScaleDiv kd(ks), vd(vs);
    while (true) {
#pragma unroll
      for (int j = 0; j < GROUPS; ++j) {
        if (dst[j] < 0) {
          if (dst[j] == -2 && invalid != nullptr) atomicAdd(invalid, 1);
          continue;
        }
        if constexpr (kVec) {
          st_v4(k_cache + dst[j], rk[j].quantize(kd));
          st_v4(v_cache + dst[j], rv[j].quantize(vd));
        } else {
          float xk[16], xv[16];
          load_vals(src_k(it1), xk);
          load_vals(src_v(it1), xv);
          store_group(it1, xk, xv, kd, vd, false);
        }
      }
      base += nthreads * GROUPS;
      if (base >= total) break;
      load_stride();
    }
    return;
  }

  // ---------------------------------------------------------------- calibration
  // amax of this thread's share of the whole batch (every token, slot -1 included, as
  // the reference takes key.abs().amax() over the batch)
  float mk = 0.0f, mv = 0.0f;
  for (uint32_t i = tid0; i < total; i += nthreads) {
    Item c;
    c.t = pt_shift >= 0 ? i >> pt_shift : i / per_token;
    const uint32_t rem = i - c.t * per_token;
    c.h = gr_shift >= 0 ? rem >> gr_shift : rem / groups_per_row;
    c.g = rem - c.h * groups_per_row;
    float xk[16], xv[16];
    if constexpr (kVec) {
      Raw16<T> a, b;
      a.load(src_k(c));
      b.load(src_v(c));
      a.get(xk);
      b.get(xv);
    } else {
      load_vals(src_k(c), xk);
      load_vals(src_v(c), xv);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      mk = amax_step(mk, fabsf(xk[j]));
      mv = amax_step(mv, fabsf(xv[j]));
    }
  }
  unsigned int bk = __float_as_uint(mk), bv = __float_as_uint(mv);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    bk = max(bk, __shfl_xor_sync(0xffffffffu, bk, o));
    bv = max(bv, __shfl_xor_sync(0xffffffffu, bv, o));
  }
  __shared__ unsigned int wk[kStoreThreads / 32], wv[kStoreThreads / 32];
  __shared__ bool is_last;
  __shared__ float new_scale[2];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    wk[wid] = bk;
    wv[wid] = bv;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int a = 0, b = 0;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) {
      a = max(a, wk[w]);
      b = max(b, wv[w]);
    }
    if (need_k) atomicMax(&work->amax_bits[0], a);
    if (need_v) atomicMax(&work->amax_bits[1], b);
    __threadfence();
    const unsigned int prev = atomicAdd(&work->arrived[0], 1u);
    is_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int fk = atomicExch(&work->amax_bits[0], 0u);
    const unsigned int fv = atomicExch(&work->amax_bits[1], 0u);
    atomicExch(&work->arrived[0], 0u);
    float sk = ks, sv = vs;
    if (need_k) {
      sk = torch_fp8_scale<T>(__uint_as_float(fk));
      *k_scale = sk;
    }
    if (need_v) {
      sv = torch_fp8_scale<T>(__uint_as_float(fv));
      *v_scale = sv;
    }
    new_scale[0] = sk;
    new_scale[1] = sv;
  }
  __syncthreads();
  const ScaleDiv kd(new_scale[0]), vd(new_scale[1]);
  // This CTA stores the batch. One group per thread in flight keeps the kernel at the
  // steady state's 64 registers; the single-CTA store is paid on the first call only.
  for (uint32_t i = threadIdx.x; i < total; i += blockDim.x) {
    Item c;
    locate(i, c);
    float xk[16], xv[16];
    if constexpr (kVec) {
      Raw16<T> a, b;
      a.load(src_k(c));
      b.load(src_v(c));
      a.get(xk);
      b.get(xv);
    } else {
      load_vals(src_k(c), xk);
      load_vals(src_v(c), xv);
    }
    store_group(c, xk, xv, kd, vd, true);
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

// One group of LPR lanes (a power of two >= head_dim / 16) per (token, kv head) row; each
// lane group takes ROWS rows per loop step, ROWS rows apart in the grid's row order (the
// grid covers rows / ROWS groups). Each lane loads 16 elements of K and of V of every
// row first (all 4 * ROWS * 16-byte loads in flight), then per row and tensor the group
// reduces the amax with shuffles and each lane writes its 16 quantised bytes; lane 0 of
// the group writes the row's scales. The loop is warp-uniform so that every lane takes
// part in the shuffles.
template <typename T, bool kInt8, typename SlotT, int ROWS>
__global__ void __launch_bounds__(kStoreThreads, 4)
store_kv_pth_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                    int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                    uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                    float* __restrict__ k_scales, float* __restrict__ v_scales,
                    const SlotT* __restrict__ slots, int64_t num_slots, int64_t num_tokens,
                    int num_heads, int groups_per_row, int lpr_shift, bool vec,
                    int32_t* invalid) {
  pdl_trigger();  // a dependent decode may begin its prologue now
  const int lpr = 1 << lpr_shift;
  const int lane = threadIdx.x & 31;
  const int sub = lane & (lpr - 1);
  const int64_t rows = num_tokens * num_heads;
  const int64_t groups = ((int64_t)gridDim.x * blockDim.x) >> lpr_shift;  // lane groups
  const int64_t step = groups * ROWS;
  for (int64_t r0 = ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) >> lpr_shift;
       r0 < rows; r0 += step) {
    int64_t slot[ROWS], dst[ROWS];
    bool ok[ROWS], has[ROWS];
    int hh[ROWS];
    const uint8_t* src[ROWS][2];
    Raw16<T> raw[ROWS][2];  // vector form: converted only when the row is processed
#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      const int64_t row = r0 + (lane >> lpr_shift) + (int64_t)j * groups;
      int64_t t = 0;
      int h = 0;
      slot[j] = -1;
      if (row < rows) {
        t = row / num_heads;
        h = (int)(row - t * num_heads);
        slot[j] = load_index(slots, t);
        if (slot[j] >= num_slots && h == 0 && sub == 0 && invalid != nullptr) atomicAdd(invalid, 1);
      }
      hh[j] = h;
      ok[j] = row < rows && slot[j] >= 0 && slot[j] < num_slots;
      has[j] = ok[j] && sub < groups_per_row;
      dst[j] = ((slot[j] * num_heads + h) * groups_per_row + sub) * 16;
      const int64_t src_off = (int64_t)sub * 16 * (int64_t)sizeof(T);
      src[j][0] = key + t * k_st + h * k_sh + src_off;
      src[j][1] = value + t * v_st + h * v_sh + src_off;
      if (has[j] && vec) {
        raw[j][0].load(src[j][0]);
        raw[j][1].load(src[j][1]);
      }
    }
#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        float x[16];
        if (has[j]) {
          if (vec) raw[j][which].get(x);
          else load16<T>(src[j][which], false, x);
        }
        float amax = 0.0f;
        int nan = 0;
        if (has[j]) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float a = fabsf(x[e]);
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
        if (has[j]) {
          uint4 packed;
          if (kInt8) {
            const float inv = 1.0f / scale;
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[i] = (uint32_t)(uint8_t)quantize_int8(x[4 * i + 0], inv) |
                     ((uint32_t)(uint8_t)quantize_int8(x[4 * i + 1], inv) << 8) |
                     ((uint32_t)(uint8_t)quantize_int8(x[4 * i + 2], inv) << 16) |
                     ((uint32_t)(uint8_t)quantize_int8(x[4 * i + 3], inv) << 24);
            packed = make_uint4(w[0], w[1], w[2], w[3]);
          } else {
            packed = quantize16(x, ScaleDiv(scale));
          }
          st_v4((which == 0 ? k_cache : v_cache) + dst[j], packed);
        }
        if (ok[j] && sub == 0) (which == 0 ? k_scales : v_scales)[slot[j] * num_heads + hh[j]] = scale;
      }
    }
  }
}

// -------------------------------------------------------------------- FP8 calibration

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
  const int64_t chunks = vec ? num_tokens * num_heads * (row_bytes / 16) : 0;
  if (vec && chunks < ((int64_t)1 << 31)) {
    const uint32_t row_chunks = (uint32_t)(row_bytes / 16);
    const int per = per_thread_items(chunks);
    const int grid = sm_multiple(grid_for((chunks + per - 1) / per, kStoreThreads));
    const int pt_shift = log2_if_pow2((int64_t)num_heads * row_chunks);
    const int rc_shift = log2_if_pow2(row_chunks);
#define MKV_COPY(C)                                                                            \
  store_kv_copy_kernel<SlotT, C><<<grid, kStoreThreads, 0, stream>>>(                         \
      (const uint8_t*)key, (const uint8_t*)value, k_st * eb, k_sh * eb, v_st * eb, v_sh * eb, \
      (uint8_t*)k_cache, (uint8_t*)v_cache, slots, num_slots, (uint32_t)chunks,               \
      (uint32_t)num_heads, row_chunks, pt_shift, rc_shift, invalid)
    if (per == 4) MKV_COPY(4);
    else if (per == 2) MKV_COPY(2);
    else MKV_COPY(1);
#undef MKV_COPY
  } else if (vec) {
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
                     float* k_scale, float* v_scale, int64_t num_slots,
                     const SlotT* slots, int64_t num_tokens, int num_heads, int head_dim,
                     CalibWork* work, int32_t* invalid, cudaStream_t stream) {
  const int64_t eb = sizeof(T);
  const bool vec = aligned16(key) && aligned16(value) && ((k_st * eb) % 16 == 0) &&
                   ((k_sh * eb) % 16 == 0) && ((v_st * eb) % 16 == 0) &&
                   ((v_sh * eb) % 16 == 0);
  const int groups = head_dim / 16;
  const int64_t total = num_tokens * num_heads * groups;
  if (total >= ((int64_t)1 << 31)) {  // beyond 32-bit group indices: the two-kernel form
    if (work != nullptr) {
      int blocks = grid_for(total, kStoreThreads);
      if (blocks > kNumSMs * 4) blocks = kNumSMs * 4;
      fp8_calibrate_kernel<T><<<dim3(blocks, 2), kStoreThreads, 0, stream>>>(
          (const uint8_t*)key, (const uint8_t*)value, k_st * eb, k_sh * eb, v_st * eb, v_sh * eb,
          num_tokens, num_heads, head_dim, vec, k_scale, v_scale, work);
    }
    const int grid = grid_for(total, kStoreThreads);
    store_kv_fp8_kernel<T, SlotT><<<grid, kStoreThreads, 0, stream>>>(
        (const uint8_t*)key, (const uint8_t*)value, k_st * eb, k_sh * eb, v_st * eb, v_sh * eb,
        (uint8_t*)k_cache, (uint8_t*)v_cache, k_scale, v_scale, slots, num_slots, num_tokens,
        num_heads, groups, vec, invalid);
    return cuda_status(cudaGetLastError(), "store_kvcache_fp8 launch");
  }
  // two groups per thread for 16-bit keys (fp32 keys would spill at the 64-register cap)
  const int per = (vec && sizeof(T) == 2 && per_thread_items(total) >= 2) ? 2 : 1;
  const int grid = sm_multiple(grid_for((total + per - 1) / per, kStoreThreads));
  const int pt_shift = log2_if_pow2((int64_t)num_heads * groups);
  const int gr_shift = log2_if_pow2(groups);
#define MKV_FP8(G, V)                                                                            \
  store_kv_fp8_calib_kernel<T, SlotT, G, V><<<grid, kStoreThreads, 0, stream>>>(                \
      (const uint8_t*)key, (const uint8_t*)value, k_st * eb, k_sh * eb, v_st * eb, v_sh * eb,   \
      (uint8_t*)k_cache, (uint8_t*)v_cache, k_scale, v_scale, slots, num_slots, (uint32_t)total, \
      (uint32_t)num_heads, (uint32_t)groups, pt_shift, gr_shift, work, invalid)
  if (!vec) {
    MKV_FP8(1, false);
  } else if constexpr (sizeof(T) == 2) {
    if (per == 2) MKV_FP8(2, true);
    else MKV_FP8(1, true);
  } else {
    MKV_FP8(1, true);
  }
#undef MKV_FP8
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
  // One row per lane group: two rows per group (the kernel's ROWS) keeps as many bytes
  // in flight per SM but needs ~90 registers, so half as many CTAs fit.
  const int64_t lanes = (num_tokens * num_heads) << lpr_shift;
  const int grid = sm_multiple(grid_for(lanes, kStoreThreads));
  store_kv_pth_kernel<T, kInt8, SlotT, 1><<<grid, kStoreThreads, 0, stream>>>(
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

namespace mkv {
namespace {
int store_fp8_impl(const char* fn, const void* key, const void* value, int64_t key_stride_token,
                   int64_t key_stride_head, int64_t value_stride_token, int64_t value_stride_head,
                   void* k_cache, void* v_cache, float* k_scale, float* v_scale,
                   int64_t num_blocks, int32_t block_size, const void* slot_mapping,
                   int32_t slot_index_type, int64_t num_tokens, int32_t num_kv_heads,
                   int32_t head_dim, int32_t dtype, void* calib_work, int32_t* invalid_count,
                   void* stream) {
  clear_error();
  int st = check_common(key, value, k_cache, v_cache, slot_mapping, slot_index_type, num_blocks,
                        block_size, num_tokens, num_kv_heads, head_dim, fn);
  if (st != MKV_OK) return st;
  if (head_dim % 16 != 0)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: head_dim must be a multiple of 16 (got %d)", fn,
                     head_dim);
  if (!k_scale || !v_scale)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: null scale pointer", fn);
  if ((((uintptr_t)k_cache) & 15u) || (((uintptr_t)v_cache) & 15u))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: caches must be 16-byte aligned", fn);
  if (calib_work != nullptr && ((uintptr_t)calib_work & 7u) != 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: calib_work must be 8-byte aligned", fn);
  if (num_tokens == 0) return MKV_OK;
  const int64_t num_slots = num_blocks * block_size;
  cudaStream_t s = (cudaStream_t)stream;
  CalibWork* work = (CalibWork*)calib_work;
  const bool i64 = slot_index_type == MKV_INDEX_I64;
#define MKV_STORE8(T)                                                                          \
  return i64 ? launch_store_fp8<T, int64_t>(key, value, key_stride_token, key_stride_head,     \
                                            value_stride_token, value_stride_head, k_cache,    \
                                            v_cache, k_scale, v_scale, num_slots,              \
                                            (const int64_t*)slot_mapping, num_tokens,          \
                                            num_kv_heads, head_dim, work, invalid_count, s)    \
             : launch_store_fp8<T, int32_t>(key, value, key_stride_token, key_stride_head,     \
                                            value_stride_token, value_stride_head, k_cache,    \
                                            v_cache, k_scale, v_scale, num_slots,              \
                                            (const int32_t*)slot_mapping, num_tokens,          \
                                            num_kv_heads, head_dim, work, invalid_count, s)
  switch (dtype) {
    case MKV_DTYPE_F32: MKV_STORE8(float);
    case MKV_DTYPE_F16: MKV_STORE8(f16);
    case MKV_DTYPE_BF16: MKV_STORE8(bf16);
    default:
      return set_error(MKV_ERR_UNSUPPORTED, "%s: key dtype must be f32, f16 or bf16 (got %d)", fn,
                       dtype);
  }
#undef MKV_STORE8
}
}  // namespace
}  // namespace mkv

extern "C" int mkv_store_kvcache_fp8(const void* key, const void* value,
                                     int64_t key_stride_token, int64_t key_stride_head,
                                     int64_t value_stride_token, int64_t value_stride_head,
                                     void* k_cache, void* v_cache, const float* k_scale,
                                     const float* v_scale, int64_t num_blocks,
                                     int32_t block_size, const void* slot_mapping,
                                     int32_t slot_index_type, int64_t num_tokens,
                                     int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                                     int32_t* invalid_count, void* stream) {
  // without calibration scratch the kernel only reads the scales
  return store_fp8_impl("mkv_store_kvcache_fp8", key, value, key_stride_token, key_stride_head,
                        value_stride_token, value_stride_head, k_cache, v_cache,
                        const_cast<float*>(k_scale), const_cast<float*>(v_scale), num_blocks,
                        block_size, slot_mapping, slot_index_type, num_tokens, num_kv_heads,
                        head_dim, dtype, nullptr, invalid_count, stream);
}

extern "C" int mkv_store_kvcache_fp8_calibrating(
    const void* key, const void* value, int64_t key_stride_token, int64_t key_stride_head,
    int64_t value_stride_token, int64_t value_stride_head, void* k_cache, void* v_cache,
    float* k_scale, float* v_scale, int64_t num_blocks, int32_t block_size,
    const void* slot_mapping, int32_t slot_index_type, int64_t num_tokens, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype, void* calib_work, int32_t* invalid_count, void* stream) {
  return store_fp8_impl("mkv_store_kvcache_fp8_calibrating", key, value, key_stride_token,
                        key_stride_head, value_stride_token, value_stride_head, k_cache, v_cache,
                        k_scale, v_scale, num_blocks, block_size, slot_mapping, slot_index_type,
                        num_tokens, num_kv_heads, head_dim, dtype, calib_work, invalid_count,
                        stream);
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
