// Shared device/host helpers for libmkv: element types, conversions, cp.async and
// ldmatrix/mma wrappers, error reporting. sm_100a only.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/mkv.h"

namespace mkv {

// ---------------------------------------------------------------- error reporting
// Records a printf-style message for mkv_last_error() and returns `status`.
int set_error(int status, const char* fmt, ...);
void clear_error();
// Maps a CUDA error to MKV_ERR_CUDA with a message naming `what`.
int cuda_status(cudaError_t err, const char* what);

// ---------------------------------------------------------------- per-context state
// Kernel attributes and module symbols belong to a CUDA context, not to a device: a
// caller may make its own driver-API context current, and cudaDeviceReset replaces the
// primary context. Anything cached across calls is therefore keyed on the current
// context's unique ID (cuCtxGetId; IDs are never reused within a process).
// *id = 0 when no context is current on the calling thread.
int current_context_id(unsigned long long* id);
// cudaFuncSetAttribute(func, MaxDynamicSharedMemorySize, bytes), once per (kernel,
// context, size); a no-op for bytes <= 48 KB.
int ensure_dynamic_smem(const void* func, int bytes, const char* what);

// ---------------------------------------------------------------- element types
using bf16 = __nv_bfloat16;
using f16 = __half;
using fp8 = __nv_fp8_e4m3;

template <typename T> struct ElemBytes { static constexpr int value = sizeof(T); };

inline int dtype_bytes(int dtype) {
  switch (dtype) {
    case MKV_DTYPE_F32: return 4;
    case MKV_DTYPE_F16: return 2;
    case MKV_DTYPE_BF16: return 2;
    case MKV_DTYPE_FP8_E4M3: return 1;
    default: return 0;
  }
}

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(f16 x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(fp8 x) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(x.__x, __NV_E4M3);
  return __half2float(__half(h));
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ f16 from_f32<f16>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ bf16 from_f32<bf16>(float x) { return __float2bfloat16_rn(x); }

// Round a float to the precision of T and back (the arithmetic dtype of torch ops on T).
template <typename T> __device__ __forceinline__ float round_through(float x) {
  return to_f32(from_f32<T>(x));
}

// Saturating round-to-nearest-even float -> e4m3 (the CUDA fp8 conversion API).
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float to_f32(int8_t x) { return (float)x; }

// Two int8 bytes (low byte = element 0) -> half2 (x = element 0), exact: each byte,
// sign-flipped to 0..255, becomes the low mantissa bits of f16 1024 (0x6400), and
// 1152 = 1024 + 128 is subtracted (f16 is exact on 1024..2047).
__device__ __forceinline__ uint32_t s8x2_to_f16x2(uint16_t v) {
  const uint32_t w = __byte_perm((uint32_t)v, 0x64006400u, 0x7150) ^ 0x00800080u;
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&w), __half2(__half(1152.0f), __half(1152.0f)));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// Two e4m3 bytes (low byte = element 0) -> half2 (x = element 0), exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v, __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

// Four e4m3 bytes of w (byte i = element i) -> two half2 words (elements 0,1 and 2,3),
// exact: one cvt.rn.f16x2.e4m3x2 per pair, on the halves of w.
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& h01, uint32_t& h23) {
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "mov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h01), "=r"(h23)
      : "r"(w));
}

// ---------------------------------------------------------------- index loads
template <typename I> __device__ __forceinline__ int64_t load_index(const I* p, int64_t i) {
  return (int64_t)__ldg(p + i);
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while the previous
// kernel on its stream still runs; pdl_wait() returns once that kernel has completed and
// its memory operations are visible (at once when the launch had no such dependency).
// pdl_trigger() lets the next kernel launch as soon as every CTA of this one has issued
// it; without it the next kernel starts when this one ends.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// ---------------------------------------------------------------- memory ops
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// 16-byte cp.async global->shared; src_bytes = 0 zero-fills the destination
// without reading global memory.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
// 4-byte cp.async (L1-allocating form, the only one for sizes below 16); src_bytes 0
// zero-fills the destination.
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// Two 16x16 matrices of 8-bit elements, transposed (sm_100a): lanes 0-15 give the row
// addresses of the first, 16-31 those of the second. Lane l receives, per matrix, the
// column l / 4 (first register) and l / 4 + 8 (second) at rows 4 (l % 4) .. 4 (l % 4) + 3,
// one row per byte, lowest row in the lowest byte: the A fragment of an 8-bit
// m16n8k32 MMA whose A is stored K-major.
__device__ __forceinline__ void ldmatrix_b8_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                     uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16) * B(16x8) + D, fp32 accumulate.
template <typename T> struct Mma;
template <> struct Mma<bf16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct Mma<f16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

// 2^x by the hardware approximation (ex2.approx.ftz: relative error ~2^-22, 2^-inf = +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one sm_100 instruction.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Two fp32 values in one 64-bit register pair, for the packed sm_100 fp32 instructions.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Pack two floats into a 32-bit pair of T (x = low half).
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<bf16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<f16>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

constexpr int kNumSMs = 148;  // B200

}  // namespace mkv
