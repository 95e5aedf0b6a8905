// Tensor-parallel all-reduce fused with the residual add and RMSNorm that follow it.
//
// Reference: RowParallelLinear.forward (src/myvllm/layers/linear.py:222-225) all-reduces
// the o_proj / down_proj partial products with NCCL, and the next LayerNorm call
// (src/myvllm/layers/layernorm.py:17-27, residual_rms_forward) computes
//   s = x + residual;  out = s / sqrt(mean(s^2) + eps) * weight;  residual <- s.
// Here one kernel does all of it over NVLink peer memory (one-shot). Every rank owns two
// exchange buffers and a flag array that the other ranks map with CUDA IPC. The call's
// epoch lives on the device (state[0], advanced by the last block of each call), so the
// call can be captured in a CUDA graph; call e uses exchange buffer e % 2. Each block of
// each rank
//   1. copies its rows of the caller's partial into its exchange buffer, then stores the
//      epoch into its slot of every rank's flags (release, system scope) and waits,
//      bounded, until every rank's same block has stored it into this rank's (acquire);
//   2. for its rows, loads the N partials with 16-byte peer loads (L2 only), sums them
//      in fp32 in rank order (so every rank computes bit-identical results), rounds to
//      the data type, adds the residual (rounded again: the residual output) and
//      normalises.
// A block rewrites exchange buffer e % 2 at call e + 2 only after every rank's same
// block has entered call e + 1, so after it finished reading that buffer at call e: no
// exit barrier is needed. A wait that runs out (a rank that died or never came) sets
// the error flag and the block skips the rest. No multicast objects and no NVLS: plain
// peer loads and stores.
// world_size 1 (or a partial already summed by NCCL) is the same kernel without the
// exchange.
#include <cstdint>
#include <cstring>
#include <type_traits>
#include <cuda_runtime.h>

#include "mkv.h"
#include "mkv_common.cuh"

namespace mkv {
namespace {

constexpr int kArMaxRanks = 8;
constexpr int kArThreads = 128;

struct ArParams {
  const void* partial;                 // this rank's partial (num_tokens x hidden)
  void* peer_bufs[kArMaxRanks];        // each rank's two exchange buffers, buf_stride bytes apart
  int64_t buf_stride;
  uint32_t* peer_flags[kArMaxRanks];   // each rank's flags: [block][source rank]
  int rank, world;
  uint32_t* state;                     // this rank's: [0] epoch of the last call, [1] blocks done
  const void* residual;  // (num_tokens, hidden), added to the sum; may be null
  void* residual_out;    // (num_tokens, hidden), receives the sum; may be null or == residual
  const void* weight;    // (hidden,)
  void* out;             // (num_tokens, hidden)
  int64_t num_tokens;
  int hidden;
  float eps;
  int* error_flag;       // set to 1 when a wait times out
  long long timeout_cycles;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// kCg: load through L2 only (ld.global.cg), for other ranks' partials: L1 is not coherent
// with their writes.
template <typename T, bool kCg = false>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  const uint4 v = kCg ? __ldcg(reinterpret_cast<const uint4*>(p)) : *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if constexpr (std::is_same<T, bf16>::value) {
      const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
      f[2 * j] = x.x;
      f[2 * j + 1] = x.y;
    } else {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      f[2 * j] = x.x;
      f[2 * j + 1] = x.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]) {
  uint4 v;
  v.x = pack2<T>(f[0], f[1]);
  v.y = pack2<T>(f[2], f[3]);
  v.z = pack2<T>(f[4], f[5]);
  v.w = pack2<T>(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = v;
}

// Rounds through T, as the reference's bf16/f16 tensor add does.
template <typename T>
__device__ __forceinline__ float round_to(float x) {
  if constexpr (std::is_same<T, bf16>::value) return __bfloat162float(__float2bfloat16_rn(x));
  else return __half2float(__float2half_rn(x));
}

// One block per group of rows; kChunks 16-byte chunks of a row per thread (hidden <= 8 *
// kArThreads * kChunks).
template <typename T, int kChunks>
__global__ void __launch_bounds__(kArThreads) allreduce_residual_rmsnorm_kernel(const ArParams p) {
  __shared__ float red[kArThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.state) + 1;
  const int64_t par = (epoch & 1) * p.buf_stride;
  const int vec = p.hidden / 8;  // 16-byte chunks per row
  bool ok = true;
  if (p.world > 1) {
    // this block's rows of the partial -> this rank's exchange buffer of the call
    uint4* own = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.peer_bufs[p.rank]) + par);
    const uint4* src = reinterpret_cast<const uint4*>(p.partial);
    for (int64_t row = blockIdx.x; row < p.num_tokens; row += gridDim.x)
      for (int c = tid; c < vec; c += kArThreads) own[row * vec + c] = src[row * vec + c];
    __syncthreads();
    if (tid < p.world) {
      st_release_sys(p.peer_flags[tid] + blockIdx.x * kArMaxRanks + p.rank, epoch);
      const uint32_t* f = p.peer_flags[p.rank] + blockIdx.x * kArMaxRanks + tid;
      const long long t0 = clock64();
      // epochs only grow: a peer already in a later call has stored a larger one
      while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
        if (clock64() - t0 > p.timeout_cycles) {
          ok = false;
          break;
        }
      }
    }
    ok = __syncthreads_and(ok) != 0;
  }
  // ---- rows of this block
  const T* w = reinterpret_cast<const T*>(p.weight);
  for (int64_t row = blockIdx.x; ok && row < p.num_tokens; row += gridDim.x) {
    float s[kChunks][8];
    float sq = 0.0f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int col = (c * kArThreads + tid) * 8;
      if (col >= p.hidden) continue;
      const int64_t off = row * p.hidden + col;
#pragma unroll
      for (int e = 0; e < 8; ++e) s[c][e] = 0.0f;
      for (int r = 0; r < p.world; ++r) {  // rank order: identical sums on every rank
        float x[8];
        if (r == p.rank || p.world == 1)
          load8(reinterpret_cast<const T*>(p.partial) + off, x);
        else
          load8<T, true>(reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(p.peer_bufs[r]) + par) + off, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) s[c][e] += x[e];
      }
      if (p.world > 1) {
#pragma unroll
        for (int e = 0; e < 8; ++e) s[c][e] = round_to<T>(s[c][e]);  // the all-reduced x
      }
      if (p.residual != nullptr) {
        float x[8];
        load8(reinterpret_cast<const T*>(p.residual) + off, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) s[c][e] = round_to<T>(s[c][e] + x[e]);
      }
      if (p.residual_out != nullptr) store8(reinterpret_cast<T*>(p.residual_out) + off, s[c]);
#pragma unroll
      for (int e = 0; e < 8; ++e) sq = fmaf(s[c][e], s[c][e], sq);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int k = 0; k < kArThreads / 32; ++k) tot += red[k];
    __syncthreads();  // red is reused by the next row
    const float inv = rsqrtf(tot / (float)p.hidden + p.eps);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int col = (c * kArThreads + tid) * 8;
      if (col >= p.hidden) continue;
      float wv[8], y[8];
      load8(w + col, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = s[c][e] * inv * wv[e];
      store8(reinterpret_cast<T*>(p.out) + row * p.hidden + col, y);
    }
  }
  if (!ok && tid == 0) atomicExch(p.error_flag, 1);
  // the last block of the call publishes its epoch for the next call
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.state + 1, 1u) == gridDim.x - 1) {
      p.state[1] = 0;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(p.state) = epoch;
    }
  }
}

template <typename T>
int launch_ar(const ArParams& p, cudaStream_t s, int blocks) {
  const int chunks = (p.hidden / 8 + kArThreads - 1) / kArThreads;
  if (chunks <= 1) allreduce_residual_rmsnorm_kernel<T, 1><<<blocks, kArThreads, 0, s>>>(p);
  else if (chunks <= 2) allreduce_residual_rmsnorm_kernel<T, 2><<<blocks, kArThreads, 0, s>>>(p);
  else if (chunks <= 4) allreduce_residual_rmsnorm_kernel<T, 4><<<blocks, kArThreads, 0, s>>>(p);
  else allreduce_residual_rmsnorm_kernel<T, 8><<<blocks, kArThreads, 0, s>>>(p);
  return cuda_status(cudaGetLastError(), "allreduce_residual_rmsnorm launch");
}

}  // namespace
}  // namespace mkv

using namespace mkv;

extern "C" int mkv_allreduce_residual_rmsnorm(
    const void* partial, void* const* peer_bufs, int64_t buf_stride, uint32_t* const* peer_flags,
    int32_t rank, int32_t world_size, uint32_t* state, const void* residual, void* residual_out,
    const void* weight, void* out,
    int64_t num_tokens,
    int32_t hidden, int32_t dtype, float eps, int32_t* error_flag, int64_t timeout_cycles,
    void* stream) {
  clear_error();
  const char* fn = "mkv_allreduce_residual_rmsnorm";
  if (world_size < 1 || world_size > kArMaxRanks || rank < 0 || rank >= world_size)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: rank %d / world_size %d (at most %d ranks)", fn,
                     rank, world_size, kArMaxRanks);
  if (num_tokens < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > 8 * kArThreads * 8)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: hidden must be a multiple of 8, at most %d (got %d)", fn,
                     8 * kArThreads * 8, hidden);
  if (dtype != MKV_DTYPE_BF16 && dtype != MKV_DTYPE_F16)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: dtype must be bf16 or f16", fn);
  if (num_tokens == 0) return MKV_OK;
  if (!partial || !weight || !out || !state ||
      (world_size > 1 && (!peer_bufs || !peer_flags || !error_flag)))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  ArParams p;
  p.partial = partial;
  p.buf_stride = buf_stride;
  for (int r = 0; r < kArMaxRanks; ++r) {
    p.peer_bufs[r] = (r < world_size && world_size > 1) ? peer_bufs[r] : nullptr;
    p.peer_flags[r] = (r < world_size && world_size > 1) ? peer_flags[r] : nullptr;
  }
  if (world_size > 1) {
    if (buf_stride < num_tokens * hidden * (int64_t)2 || (buf_stride & 15))
      return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: exchange buffers too small or misaligned", fn);
    for (int r = 0; r < world_size; ++r)
      if (!p.peer_bufs[r] || ((uintptr_t)p.peer_bufs[r] & 15u) || !p.peer_flags[r])
        return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: rank %d buffers missing or misaligned", fn, r);
  }
  if ((uintptr_t)partial & 15u)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: partial must be 16-byte aligned", fn);
  if (((uintptr_t)out & 15u) || ((uintptr_t)weight & 15u) || ((uintptr_t)residual & 15u) ||
      ((uintptr_t)residual_out & 15u))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: out, weight and residuals must be 16-byte aligned", fn);
  p.rank = rank;
  p.world = world_size;
  p.state = state;
  p.residual = residual;
  p.residual_out = residual_out;
  p.weight = weight;
  p.out = out;
  p.num_tokens = num_tokens;
  p.hidden = hidden;
  p.eps = eps;
  p.error_flag = error_flag;
  p.timeout_cycles = timeout_cycles > 0 ? timeout_cycles : 2000000000ll;
  const int blocks = (int)(num_tokens < MKV_AR_MAX_BLOCKS ? num_tokens : MKV_AR_MAX_BLOCKS);
  cudaStream_t s = (cudaStream_t)stream;
  return dtype == MKV_DTYPE_BF16 ? launch_ar<bf16>(p, s, blocks) : launch_ar<f16>(p, s, blocks);
}

extern "C" int mkv_ipc_alloc(size_t bytes, void** ptr, void* handle_out) {
  clear_error();
  if (!ptr || !handle_out || bytes == 0) return set_error(MKV_ERR_INVALID_ARGUMENT, "mkv_ipc_alloc: bad arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_status(e, "mkv_ipc_alloc: cudaMalloc");
  e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_status(e, "mkv_ipc_alloc: cudaIpcGetMemHandle");
  }
  return MKV_OK;
}

extern "C" int mkv_ipc_free(void* ptr) {
  clear_error();
  return cuda_status(cudaFree(ptr), "mkv_ipc_free");
}

extern "C" int mkv_ipc_open(const void* handle, void** ptr) {
  clear_error();
  if (!handle || !ptr) return set_error(MKV_ERR_INVALID_ARGUMENT, "mkv_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "mkv_ipc_open");
}

extern "C" int mkv_ipc_close(void* ptr) {
  clear_error();
  return cuda_status(cudaIpcCloseMemHandle(ptr), "mkv_ipc_close");
}
