// Paged-attention decode on the 5th-generation tensor cores (tcgen05) with TMA page loads:
// a persistent, warp-specialised kernel, one CTA per SM.
//
// Semantics are those of paged_decode.cu (heart1128/mini-kvllm attention.py:517-646 and
// 953-1121): kv_head = h / (H/KVH), tokens t < min(ctx, max_blocks*block_size) on pages
// block_tables[b, t / block_size] (-1 = skip), FP8 dequantised with per-tensor scales.
//
// Roles (6 warps):
//   warp 0  producer: for every 128-token tile of a work unit, TMA loads of the K and V
//           rows (one 2D box per page segment, 128-byte swizzle) into a ring of shared
//           memory stages; segments on a missing page are zero-filled instead. Per unit it
//           writes Q^T (e4m3 hi + lo parts for FP8 pages) in the MMA operand layout.
//   warp 1  MMA issuer: one thread issues S^T = K Q^T (M = 128 tokens, N = 16 query heads,
//           K-major operands) into a TMEM S buffer and, one tile behind,
//           O^T = V^T P^T (M = 128 head_dim rows; V is MN-major straight from the TMA tile,
//           P^T comes from shared memory) into a TMEM O buffer; tcgen05.commit releases the
//           ring stage, the S/O buffers and the Q buffer through mbarriers.
//   warps 2-5  softmax: thread i owns token i of the tile for S and head_dim row i for O
//           (its TMEM lane). Per tile: read S, block max per head, exp2, write P^T; then
//           fold the previous tile's O into register accumulators.
// FP8: P is quantised to e4m3 hi + lo relative to the tile's own reference
// q_ref = max(tile max, running max - 24) scaled by 2^8, so small weights keep their
// precision; the factor 2^(q_ref - 8 - m) is applied when O is accumulated.
// A work unit is (sequence, kv head, head group, split of <= chunk tokens); CTAs walk the
// units with a fixed stride; the epilogue writes the output directly or stores partials
// that the last split of the (sequence, kv head) merges (arrival counters), as in
// paged_decode.cu.
//
// Every mbarrier wait is bounded (sm100::kWaitCycles). On a timeout the thread raises a
// CTA abort flag that all roles poll; they leave their loops, the producer waits (bounded)
// for its TMA loads in flight, the MMA thread for its MMAs, and TMEM is freed.
#include <cuda.h>

#include "mkv_common.cuh"
#include "paged_decode_tc05.cuh"
#include "sm100.cuh"

namespace mkv {
namespace tc05 {

using namespace sm100;

#ifdef MKV_TC05_TRACE
// Debug-only event timeline of CTA 0: [event][tile] global-timer stamps.
constexpr int kTraceTiles = 256;
__device__ unsigned long long g_trace[8][kTraceTiles];
__device__ __forceinline__ void trace(int ev, int64_t tile) {
  if (blockIdx.x == 0 && tile < kTraceTiles) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_trace[ev][tile] = t;
  }
}
#define MKV_TRACE(ev, tile) trace(ev, tile)
#else
#define MKV_TRACE(ev, tile)
#endif

constexpr int kTile = 128;       // tokens per tile (MMA M of S^T)
constexpr int kD = 128;          // head_dim
constexpr int kN = 16;           // query heads per unit (MMA N), padded
constexpr int kThreads = 192;    // 6 warps
constexpr int kTmemCols = 64;    // S[2] and O[2], 16 columns each
constexpr int kMaxSplits = 128;  // same bound as the split planner



template <typename CT> struct Kind;
template <> struct Kind<bf16> {
  static constexpr bool kFp8 = false;
  static constexpr int kEB = 2, kStages = 3;
  static constexpr uint32_t kFmt = 1;
};
template <> struct Kind<f16> {
  static constexpr bool kFp8 = false;
  static constexpr int kEB = 2, kStages = 3;
  static constexpr uint32_t kFmt = 0;
};
template <> struct Kind<fp8> {
  static constexpr bool kFp8 = true;
  static constexpr int kEB = 1, kStages = 6;
  static constexpr uint32_t kFmt = 0;
};

// Shared-memory layout (byte offsets from a 1024-byte aligned base).
template <typename CT>
struct Layout {
  static constexpr int EB = Kind<CT>::kEB;
  static constexpr int STAGES = Kind<CT>::kStages;
  static constexpr int BLK = kTile * 128;          // one 128-byte column block of a tile
  static constexpr int NBLK = kD * EB / 128;       // 2 for 16-bit pages, 1 for e4m3
  static constexpr int TILE = NBLK * BLK;          // K (or V) tile
  static constexpr int STAGE = 2 * TILE;           // K + V
  static constexpr int RING = STAGES * STAGE;
  static constexpr int QSTRIDE = 4096;             // Q^T buffer: 2 x [16 rows x 128 B]
  static constexpr int Q0 = RING;
  static constexpr int PBUF = Kind<CT>::kFp8 ? 2 * kTile * 16 : kTile * kN * 2;
  static constexpr int P0 = Q0 + 2 * QSTRIDE;
  static constexpr int VALID0 = P0 + 2 * PBUF;     // [STAGES][kTile]
  static constexpr int RED0 = VALID0 + STAGES * kTile;
  static constexpr int RED_FLOATS = 2 * 4 * kN + 4 * kN + (kMaxSplits + 1) * kN + 8;
  static constexpr int BAR0 = (RED0 + RED_FLOATS * 4 + 7) / 8 * 8;
  static constexpr int NBAR = 2 * STAGES + 16;  // full/empty[S], q/s/p/o pairs, drain, consumer
  static constexpr int MISC0 = BAR0 + NBAR * 8;  // tmem base, abort flag, merge flag
  static constexpr int BYTES = MISC0 + 16 + 1024;
};

__device__ __forceinline__ int64_t load_ctx(const Params& p, int seq) {
  return p.ctx_i64 ? (int64_t)__ldg((const int64_t*)p.ctx + seq)
                   : (int64_t)__ldg((const int32_t*)p.ctx + seq);
}

struct Unit {
  int seq, kvh, hg, split, begin, end, active, ntiles, h0, nh;
};

// Work unit u: the splits of one (sequence, kv head, head group) are consecutive units.
__device__ __forceinline__ Unit decode_unit(const Params& p, int64_t u) {
  Unit w;
  w.split = (int)(u % p.num_splits);
  int64_t r = u / p.num_splits;
  w.hg = (int)(r % p.head_groups);
  r /= p.head_groups;
  w.kvh = (int)(r % p.num_kv_heads);
  w.seq = (int)(r / p.num_kv_heads);
  const int64_t ctx = load_ctx(p, w.seq);
  const int64_t cap = (int64_t)p.max_blocks * p.block_size;
  int64_t eff = ctx < cap ? ctx : cap;
  if (eff < 0) eff = 0;
  w.active = eff > 0 ? (int)((eff + p.chunk - 1) / p.chunk) : 1;
  w.begin = w.split * p.chunk;
  w.end = (int)((int64_t)w.begin + p.chunk < eff ? (int64_t)w.begin + p.chunk : eff);
  w.ntiles = w.end > w.begin ? (w.end - w.begin + kTile - 1) / kTile : 0;
  w.h0 = w.kvh * p.group + w.hg * p.heads_per_cta;
  w.nh = min(p.heads_per_cta, p.group - w.hg * p.heads_per_cta);
  return w;
}

__device__ __forceinline__ int page_of(const Params& p, int seq, int blk, bool count) {
  const int64_t idx = (int64_t)seq * p.bt_sb + blk;
  const int64_t page = p.bt_i64 ? (int64_t)__ldg((const int64_t*)p.bt + idx)
                                : (int64_t)__ldg((const int32_t*)p.bt + idx);
  if (page >= 0 && page < p.num_blocks) return (int)page;
  if (page != -1 && count && p.invalid != nullptr) atomicAdd(p.invalid, 1);
  return -1;
}

// Barrier among the 4 softmax warps only (the producer and MMA warps run on), built on
// an mbarrier so that the wait is bounded like every other wait in the kernel. Each call
// completes one phase; `calls` counts the calls of this thread.
__device__ __forceinline__ bool consumer_sync(uint64_t* cbar, uint32_t& calls,
                                             const volatile int* abort) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(cbar);
  const bool ok = mbar_wait(cbar, calls & 1, abort);
  ++calls;
  __syncwarp();
  return ok;
}

// Power-of-two FP8 query scale from max |q| over the unit's heads (max |q| * qs lies in
// [128, 256)); the producer and the softmax warps derive it identically.
__device__ __forceinline__ float fp8_query_scale(float qmax) {
  float qs = 1.0f;
  if (qmax > 0.0f && isfinite(qmax)) {
    int ex;
    frexpf(qmax, &ex);
    qs = ldexpf(1.0f, 8 - ex);
  }
  return qs;
}

// e4m3 bytes of x (hi) and of the residual x - hi (lo).
__device__ __forceinline__ void split_e4m3(float x, uint32_t& hi, uint32_t& lo) {
  const uint8_t h = f32_to_e4m3(x);
  fp8 hv;
  hv.__x = h;
  hi = h;
  lo = f32_to_e4m3(x - to_f32(hv));
}

template <typename QT, typename CT>
__global__ void __launch_bounds__(kThreads, 1)
paged_decode_tc05_kernel(const Params p, const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap) {
  using L = Layout<CT>;
  constexpr bool kFp8 = Kind<CT>::kFp8;
  constexpr int STAGES = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR0);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* qfull = bars + 2 * STAGES;
  uint64_t* qempty = qfull + 2;
  uint64_t* sfull = qempty + 2;
  uint64_t* sfree = sfull + 2;
  uint64_t* pfull = sfree + 2;
  uint64_t* ofull = pfull + 2;
  uint64_t* ofree = ofull + 2;
  uint64_t* drain = ofree + 2;
  uint64_t* cbar = drain + 1;
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + L::MISC0);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC0 + 4);
  volatile int* merge_flag = reinterpret_cast<volatile int*>(smem + L::MISC0 + 8);
  uint8_t* valid = smem + L::VALID0;
  float* red = reinterpret_cast<float*>(smem + L::RED0);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&qfull[b], 1);
      mbar_init(&qempty[b], 1);
      mbar_init(&sfull[b], 1);
      mbar_init(&sfree[b], 4);
      mbar_init(&pfull[b], 4);
      mbar_init(&ofull[b], 1);
      mbar_init(&ofree[b], 4);
    }
    mbar_init(drain, 1);
    mbar_init(cbar, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_base_s, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_base_s;

  if (warp == 0) {
    // ================================================================ producer
    if (lane == 0) {
      tma_prefetch_map(&kmap);
      tma_prefetch_map(&vmap);
    }
    int64_t T = 0;  // tiles issued
    int U = 0;      // units with tiles
    const int seg_rows = p.block_size < kTile ? p.block_size : kTile;
    const int nseg = kTile / seg_rows;  // <= 16 (block_size >= 8)
    for (int64_t u = blockIdx.x; u < p.num_units && !*abort_flag; u += gridDim.x) {
      const Unit w = decode_unit(p, u);
      if (w.ntiles == 0) continue;
      const bool count = (w.kvh == 0 && w.hg == 0);
      // ---- Q^T of the unit
      const int qb = U & 1;
      if (!mbar_wait(&qempty[qb], ((U >> 1) & 1) ^ 1, abort_flag)) { *abort_flag = 1; break; }
      uint8_t* qbuf = smem + L::Q0 + qb * L::QSTRIDE;
      const QT* qp = reinterpret_cast<const QT*>(p.q) + (int64_t)w.seq * p.q_sb;
      const int h = lane >> 1, half = lane & 1;  // lane -> head, 64-column half
      const bool real = h < w.nh;
      const QT* qrow = qp + (int64_t)(w.h0 + (real ? h : 0)) * p.q_sh + half * 64;
      if (!kFp8) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // block `half`, chunk c (8 columns)
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (real) v = *reinterpret_cast<const uint4*>(qrow + c * 8);
          *reinterpret_cast<uint4*>(qbuf + half * (kN * 128) + h * 128 + ((c ^ (h & 7)) << 4)) = v;
        }
      } else {
        float mx = 0.0f;
        if (real)
          for (int d = 0; d < 64; ++d) mx = fmaxf(mx, fabsf(to_f32(qrow[d])));
        const float qs = fp8_query_scale(warp_max(mx));
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // chunk cc = half*4 + c holds columns 16cc .. 16cc+15
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            hw[k] = lw[k] = 0u;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint32_t hb, lb;
              split_e4m3(real ? to_f32(qrow[c * 16 + k * 4 + e]) * qs : 0.0f, hb, lb);
              hw[k] |= hb << (8 * e);
              lw[k] |= lb << (8 * e);
            }
          }
          const int cc = half * 4 + c;
          const int off = h * 128 + ((cc ^ (h & 7)) << 4);
          *reinterpret_cast<uint4*>(qbuf + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(qbuf + kN * 128 + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&qfull[qb]);
      ++U;
      // ---- tiles
      for (int it = 0; it < w.ntiles; ++it, ++T) {
        const int st = (int)(T % STAGES);
        const int t0 = w.begin + it * kTile;
        // page of segment `lane` (lanes >= nseg idle)
        int seg_page = -1;
        if (lane < nseg) {
          const int ts = t0 + lane * seg_rows;
          if (ts < w.end) seg_page = page_of(p, w.seq, ts >> p.bs_shift, count);
        }
        if (!mbar_wait(&empty[st], (int)((T / STAGES) & 1) ^ 1, abort_flag)) { *abort_flag = 1; break; }
        if (lane == 0) MKV_TRACE(0, T);
        uint8_t* kt = smem + st * L::STAGE;
        uint8_t* vt = kt + L::TILE;
        uint32_t bytes = 0;
        for (int r = lane; r < kTile; r += 32) {
          const int pg = __shfl_sync(0xffffffffu, seg_page, r / seg_rows);
          valid[st * kTile + r] = (t0 + r < w.end && pg >= 0) ? 1 : 0;
        }
        for (int sgi = 0; sgi < nseg; ++sgi) {
          const int pg = __shfl_sync(0xffffffffu, seg_page, sgi);
          if (pg >= 0) {
            bytes += 2u * L::NBLK * seg_rows * 128;
          } else {  // zero this segment's K and V rows (then a proxy fence below)
            for (int b = 0; b < L::NBLK; ++b)
              for (int i = lane; i < seg_rows * 8; i += 32) {
                const int off = b * L::BLK + sgi * seg_rows * 128 + i * 16;
                *reinterpret_cast<uint4*>(kt + off) = make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(vt + off) = make_uint4(0u, 0u, 0u, 0u);
              }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        for (int sgi = 0; sgi < nseg; ++sgi) {
          const int pg = __shfl_sync(0xffffffffu, seg_page, sgi);
          if (lane == 0) {
            if (sgi == 0) mbar_arrive_expect_tx(&full[st], bytes);
            if (pg >= 0) {
              const int ts = t0 + sgi * seg_rows;
              const int y = pg * p.block_size + (ts & (p.block_size - 1));
              for (int b = 0; b < L::NBLK; ++b) {
                const int x = w.kvh * kD + b * (128 / L::EB);
                const uint32_t off = b * L::BLK + sgi * seg_rows * 128;
                tma_load_2d(smem_u32(kt + off), &kmap, x, y, &full[st]);
                tma_load_2d(smem_u32(vt + off), &vmap, x, y, &full[st]);
              }
            }
          }
        }
        __syncwarp();
      }
    }
    if (lane == 0 && *abort_flag) {  // let issued loads land before the CTA exits
      for (int64_t k = T - STAGES; k < T; ++k)
        if (k >= 0) mbar_wait(&full[k % STAGES], (int)((k / STAGES) & 1), nullptr);
    }
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    constexpr uint32_t kIdQK = instr_desc(Kind<CT>::kFmt, Kind<CT>::kFmt, 0, 0, kTile, kN);
    constexpr uint32_t kIdPV = instr_desc(Kind<CT>::kFmt, Kind<CT>::kFmt, 1, 1, kD, kN);
    int64_t T = 0;
    int U = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
      const Unit w = decode_unit(p, u);
      if (w.ntiles == 0) continue;
      const int qb = U & 1;
      ok = mbar_wait(&qfull[qb], (U >> 1) & 1, abort_flag);
      if (!ok) break;
      const uint32_t qaddr = smem_u32(smem + L::Q0 + qb * L::QSTRIDE);
      for (int it = 0; it <= w.ntiles && ok; ++it) {
        if (it < w.ntiles) {  // S^T(it) = K Q^T
          const int64_t Ti = T + it;
          const int st = (int)(Ti % STAGES), sb = (int)(Ti & 1);
          ok = mbar_wait(&full[st], (int)((Ti / STAGES) & 1), abort_flag) &&
               mbar_wait(&sfree[sb], (int)((Ti >> 1) & 1) ^ 1, abort_flag);
          if (!ok) break;
          tc_fence_after_sync();
          if (lane == 0) {
            const uint32_t kaddr = smem_u32(smem + st * L::STAGE);
            const uint32_t dS = tmem + sb * kN;
            if (!kFp8) {
#pragma unroll
              for (int k = 0; k < 8; ++k) {  // 16 columns of head_dim per MMA
                const uint64_t a = smem_desc(kaddr + (k >> 2) * L::BLK + (k & 3) * 32, 16, 1024, kLayoutSw128);
                const uint64_t b = smem_desc(qaddr + (k >> 2) * (kN * 128) + (k & 3) * 32, 16, 1024, kLayoutSw128);
                mma_f16(dS, a, b, kIdQK, k > 0);
              }
            } else {
#pragma unroll
              for (int part = 0; part < 2; ++part)  // query hi, then lo, one accumulator
#pragma unroll
                for (int k = 0; k < 4; ++k) {       // 32 columns per MMA
                  const uint64_t a = smem_desc(kaddr + k * 32, 16, 1024, kLayoutSw128);
                  const uint64_t b = smem_desc(qaddr + part * (kN * 128) + k * 32, 16, 1024, kLayoutSw128);
                  mma_f8(dS, a, b, kIdQK, (part | k) != 0);
                }
            }
            mma_commit(&sfull[sb]);
            MKV_TRACE(1, Ti);
            if (it == w.ntiles - 1) mma_commit(&qempty[qb]);
          }
          __syncwarp();
        }
        if (it > 0) {  // O^T(it-1) = V^T P^T
          const int64_t Tj = T + it - 1;
          const int st = (int)(Tj % STAGES), b2 = (int)(Tj & 1);
          ok = mbar_wait(&pfull[b2], (int)((Tj >> 1) & 1), abort_flag) &&
               mbar_wait(&ofree[b2], (int)((Tj >> 1) & 1) ^ 1, abort_flag);
          if (!ok) break;
          tc_fence_after_sync();
          if (lane == 0) {
            const uint32_t vaddr = smem_u32(smem + st * L::STAGE + L::TILE);
            const uint32_t paddr = smem_u32(smem + L::P0 + b2 * L::PBUF);
            const uint32_t dO = tmem + 2 * kN + b2 * kN;
            if (!kFp8) {
#pragma unroll
              for (int k = 0; k < kTile / 16; ++k) {  // 16 tokens per MMA
                const uint64_t a = smem_desc(vaddr + k * 2048, L::BLK, 1024, kLayoutSw128);
                const uint64_t b = smem_desc(paddr + k * 512, 256, 128, kLayoutNone);
                mma_f16(dO, a, b, kIdPV, k > 0);
              }
            } else {
#pragma unroll
              for (int part = 0; part < 2; ++part)  // P hi, then lo
#pragma unroll
                for (int k = 0; k < kTile / 32; ++k) {  // 32 tokens per MMA
                  const uint64_t a = smem_desc(vaddr + k * 4096, L::BLK, 1024, kLayoutSw128);
                  const uint64_t b = smem_desc(paddr + part * (kTile * 16) + k * 512, 128, 256, kLayoutNone);
                  mma_f8(dO, a, b, kIdPV, (part | k) != 0);
                }
            }
            mma_commit(&ofull[b2]);
            mma_commit(&empty[st]);
            MKV_TRACE(2, Tj);
          }
          __syncwarp();
        }
      }
      T += w.ntiles;
      ++U;
    }
    if (!ok) *abort_flag = 1;
    if (lane == 0) {  // every issued MMA completes before TMEM is released
      mma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
    __syncwarp();
  } else {
    // ================================================================ softmax warps
    const int ct = 32 * (warp & 3) + lane;  // TMEM lane: token of S, head_dim row of O
    const int wq = warp & 3;
    const uint32_t lane_base = (uint32_t)(32 * wq) << 16;
    float* red_max = red;                // [2][4][kN]
    float* red_sum = red + 2 * 4 * kN;   // [4][kN]
    float* wts = red_sum + 4 * kN;       // [(kMaxSplits + 1) * kN]
    const float vs = kFp8 ? __ldg(p.v_scale) : 1.0f;
    const float ksc = kFp8 ? __ldg(p.k_scale) : 1.0f;
    QT* op = reinterpret_cast<QT*>(p.out);
    int64_t T = 0;
    bool ok = true;
    uint32_t ncs = 0;  // consumer_sync calls
#define MKV_CSYNC()                                                 \
  if (!(ok = consumer_sync(cbar, ncs, abort_flag))) break;
    for (int64_t u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
      const Unit w = decode_unit(p, u);
      const bool empty_ctx = w.split == 0 && w.end <= w.begin;  // writes the NaN of 0/0
      if (w.ntiles == 0 && !empty_ctx) continue;
      float m_run[kN], l_run[kN], o_acc[kN], a_prev[kN], b_prev[kN];
#pragma unroll
      for (int h = 0; h < kN; ++h) {
        m_run[h] = -INFINITY;
        l_run[h] = 0.0f;
        o_acc[h] = 0.0f;
        a_prev[h] = 1.0f;
        b_prev[h] = 1.0f;
      }
      float sc = p.qk_scale_log2;
      if (kFp8 && w.ntiles > 0) {  // the producer's query scale, recomputed
        const QT* qp = reinterpret_cast<const QT*>(p.q) + (int64_t)w.seq * p.q_sb;
        const int hh = ct >> 3, d0 = (ct & 7) * 16;
        float mx = 0.0f;
        if (hh < w.nh)
          for (int d = 0; d < 16; ++d) mx = fmaxf(mx, fabsf(to_f32(qp[(int64_t)(w.h0 + hh) * p.q_sh + d0 + d])));
        mx = warp_max(mx);
        if (lane == 0) red_sum[wq * kN] = mx;
        MKV_CSYNC();
        mx = fmaxf(fmaxf(red_sum[0], red_sum[kN]), fmaxf(red_sum[2 * kN], red_sum[3 * kN]));
        MKV_CSYNC();
        sc = p.qk_scale_log2 * ksc / fp8_query_scale(mx);
      }
      for (int it = 0; it <= w.ntiles && ok; ++it) {
        float a_cur[kN], b_cur[kN];
        if (it < w.ntiles) {
          const int64_t Ti = T + it;
          const int st = (int)(Ti % STAGES), sb = (int)(Ti & 1);
          ok = mbar_wait(&full[st], (int)((Ti / STAGES) & 1), abort_flag) &&
               mbar_wait(&sfull[sb], (int)((Ti >> 1) & 1), abort_flag);
          if (!ok) break;
          tc_fence_after_sync();
          if (ct == 0) MKV_TRACE(3, Ti);
          float s[kN];
          tmem_ld16(tmem + lane_base + sb * kN, s);
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sfree[sb]);
          const bool v = valid[st * kTile + ct] != 0;
          float* rm = red_max + sb * 4 * kN;
#pragma unroll
          for (int h = 0; h < kN; ++h) {
            s[h] = v ? s[h] * sc : -INFINITY;
            if (h < w.nh) {
              const float mx = warp_max(s[h]);
              if (lane == 0) rm[wq * kN + h] = mx;
            }
          }
          MKV_CSYNC();
          if (ct == 0) MKV_TRACE(6, Ti);
          float pv[kN];
#pragma unroll
          for (int h = 0; h < kN; ++h) {
            pv[h] = 0.0f;
            a_cur[h] = 1.0f;
            b_cur[h] = 1.0f;
            if (h < w.nh) {
              const float tm = fmaxf(fmaxf(rm[h], rm[kN + h]), fmaxf(rm[2 * kN + h], rm[3 * kN + h]));
              const float m_new = fmaxf(m_run[h], tm);
              const float base = m_new == -INFINITY ? 0.0f : m_new;
              a_cur[h] = exp2f(m_run[h] - base);
              m_run[h] = m_new;
              const float p_run = v ? exp2f(s[h] - base) : 0.0f;  // weight in the running frame
              l_run[h] = fmaf(l_run[h], a_cur[h], p_run);
              if (!kFp8) {
                pv[h] = p_run;
              } else if (tm != -INFINITY) {
                const float qref = fmaxf(tm, m_new - 24.0f);
                pv[h] = v ? exp2f(s[h] - qref + 8.0f) : 0.0f;  // <= 256, relative to the tile
                b_cur[h] = exp2f(qref - 8.0f - base);
              }
            }
          }
          uint8_t* pbuf = smem + L::P0 + sb * L::PBUF;
          if (!kFp8) {
            uint32_t pw[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) pw[j] = pack2<QT>(pv[2 * j], pv[2 * j + 1]);
            uint8_t* dst = pbuf + (ct >> 3) * 256 + (ct & 7) * 16;  // [token group][head group][token][8 heads]
            *reinterpret_cast<uint4*>(dst) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
            *reinterpret_cast<uint4*>(dst + 128) = make_uint4(pw[4], pw[5], pw[6], pw[7]);
          } else {
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              hw[k] = lw[k] = 0u;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                uint32_t hb, lb;
                split_e4m3(pv[4 * k + e], hb, lb);
                hw[k] |= hb << (8 * e);
                lw[k] |= lb << (8 * e);
              }
            }
            uint8_t* dst = pbuf + (ct >> 3) * 128 + (ct & 7) * 16;  // [token group][token][16 heads]
            *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(dst + kTile * 16) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
          if (!v) {  // an invalid token's V row must be finite: zero it before PV reads it
            uint8_t* vrow = smem + st * L::STAGE + L::TILE + ct * 128;
#pragma unroll
            for (int b = 0; b < L::NBLK; ++b)
#pragma unroll
              for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(vrow + b * L::BLK + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pfull[sb]);
          if (ct == 0) MKV_TRACE(4, Ti);
        }
        if (it > 0) {  // fold O(it-1) into the accumulators
          const int64_t Tj = T + it - 1;
          const int b2 = (int)(Tj & 1);
          ok = mbar_wait(&ofull[b2], (int)((Tj >> 1) & 1), abort_flag);
          if (!ok) break;
          tc_fence_after_sync();
          if (ct == 0) MKV_TRACE(5, Tj);
          float o[kN];
          tmem_ld16(tmem + lane_base + 2 * kN + b2 * kN, o);
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ofree[b2]);
#pragma unroll
          for (int h = 0; h < kN; ++h) o_acc[h] = fmaf(o_acc[h], a_prev[h], o[h] * b_prev[h]);
        }
        if (it < w.ntiles) {
#pragma unroll
          for (int h = 0; h < kN; ++h) {
            a_prev[h] = a_cur[h];
            b_prev[h] = b_cur[h];
          }
        }
      }
      if (!ok) break;
      T += w.ntiles;

      // ---------------- unit epilogue (softmax warps only)
      // l: sum of the per-token partials of the 128 threads
#pragma unroll
      for (int h = 0; h < kN; ++h) {
        if (h < w.nh) {
          const float sum = warp_sum(l_run[h]);
          if (lane == 0) red_sum[wq * kN + h] = sum;
        }
      }
      MKV_CSYNC();
      float Lh[kN];
#pragma unroll
      for (int h = 0; h < kN; ++h)
        Lh[h] = (red_sum[h] + red_sum[kN + h]) + (red_sum[2 * kN + h] + red_sum[3 * kN + h]);
      MKV_CSYNC();
      const int d = ct;
      if (w.active == 1) {
#pragma unroll
        for (int h = 0; h < kN; ++h)
          if (h < w.nh) op[(int64_t)w.seq * p.o_sb + (int64_t)(w.h0 + h) * p.o_sh + d] = from_f32<QT>(o_acc[h] * vs / Lh[h]);
        continue;
      }
      const int64_t S = p.num_splits;
#pragma unroll
      for (int h = 0; h < kN; ++h) {
        if (h < w.nh) {
          const int64_t b = ((int64_t)w.seq * p.num_heads + w.h0 + h) * S + w.split;
          __stcg(p.part_acc + b * kD + d, o_acc[h]);
          if (d == 0) {
            __stcg(p.part_ml + b * 2 + 0, m_run[h]);
            __stcg(p.part_ml + b * 2 + 1, Lh[h]);
          }
        }
      }
      __threadfence();
      MKV_CSYNC();
      unsigned int* ctr = p.arrivals + ((int64_t)w.seq * p.num_kv_heads + w.kvh) * p.head_groups + w.hg;
      if (ct == 0) *merge_flag = atomicAdd(ctr, 1u) == (unsigned)(w.active - 1);
      MKV_CSYNC();
      const bool last = *merge_flag != 0;
      MKV_CSYNC();
      if (!last) continue;
      __threadfence();
      if (ct < w.nh) {
        const int64_t base = ((int64_t)w.seq * p.num_heads + w.h0 + ct) * S;
        float M = -INFINITY;
        for (int s2 = 0; s2 < w.active; ++s2) M = fmaxf(M, __ldcg(p.part_ml + (base + s2) * 2));
        const float mb = M == -INFINITY ? 0.0f : M;
        float Lsum = 0.0f;
        for (int s2 = 0; s2 < w.active; ++s2) {
          const float wgt = exp2f(__ldcg(p.part_ml + (base + s2) * 2) - mb);
          wts[s2 * kN + ct] = wgt;
          Lsum = fmaf(wgt, __ldcg(p.part_ml + (base + s2) * 2 + 1), Lsum);
        }
        wts[w.active * kN + ct] = vs / Lsum;
      }
      MKV_CSYNC();
      for (int h = 0; h < w.nh; ++h) {
        const int64_t base = ((int64_t)w.seq * p.num_heads + w.h0 + h) * S;
        float O = 0.0f;
        for (int s2 = 0; s2 < w.active; ++s2) O = fmaf(wts[s2 * kN + h], __ldcg(p.part_acc + (base + s2) * kD + d), O);
        op[(int64_t)w.seq * p.o_sb + (int64_t)(w.h0 + h) * p.o_sh + d] = from_f32<QT>(O * wts[w.active * kN + h]);
      }
      if (ct == 0) *ctr = 0u;
      MKV_CSYNC();
    }
#undef MKV_CSYNC
    if (!ok) *abort_flag = 1;
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ================================================================ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
    tried = true;
  }
  return fn;
}


bool supported(int q_dtype, int cache_dtype, int head_dim, int block_size, int heads_per_cta) {
#ifndef MKV_ENABLE_TC05
  // Off by default: on B200 this kernel measured 1.98 TB/s (bf16, config 3) against 6.05 TB/s
  // for the mma.sync kernel. With N = 16 query heads each tcgen05.mma does little work and
  // its issue-to-visible latency (~1.3 us for QK, ~1.5 us for PV, measured) keeps a 64 KB
  // tile resident for ~7 us, so the 3-stage ring holds too few tiles in flight.
  (void)q_dtype; (void)cache_dtype; (void)head_dim; (void)block_size; (void)heads_per_cta;
  return false;
#endif
  if (head_dim != kD || heads_per_cta > kN) return false;
  if (q_dtype != MKV_DTYPE_BF16 && q_dtype != MKV_DTYPE_F16) return false;
  if (cache_dtype != q_dtype && cache_dtype != MKV_DTYPE_FP8_E4M3) return false;
  if (block_size < 8 || (block_size & (block_size - 1)) != 0) return false;
  return encode_fn() != nullptr;
}

template <typename QT, typename CT>
int launch_typed(const Params& p, const CUtensorMap& km, const CUtensorMap& vm,
                 cudaStream_t stream, int device) {
  using L = Layout<CT>;
  static unsigned long long configured = 0;
  const unsigned long long bit = device < 64 ? (1ull << device) : 0ull;
  if (!bit || !(__atomic_load_n(&configured, __ATOMIC_RELAXED) & bit)) {
    cudaError_t e = cudaFuncSetAttribute(paged_decode_tc05_kernel<QT, CT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(tc05 smem)");
    if (bit) __atomic_fetch_or(&configured, bit, __ATOMIC_RELAXED);
  }
  int sms = kNumSMs;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int64_t grid = p.num_units < sms ? p.num_units : sms;
  paged_decode_tc05_kernel<QT, CT><<<(int)grid, kThreads, L::BYTES, stream>>>(p, km, vm);
  return cuda_status(cudaGetLastError(), "paged_decode_tc05 launch");
}

int launch(const Params& p, int q_dtype, int cache_dtype, const void* k_cache,
           const void* v_cache, cudaStream_t stream, int device) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return set_error(MKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const bool f8 = cache_dtype == MKV_DTYPE_FP8_E4M3;
  const int eb = f8 ? 1 : 2;
  const cuuint64_t dims[2] = {(cuuint64_t)p.num_kv_heads * kD,
                              (cuuint64_t)p.num_blocks * (cuuint64_t)p.block_size};
  const cuuint64_t strides[1] = {(cuuint64_t)p.num_kv_heads * kD * eb};
  const cuuint32_t box[2] = {(cuuint32_t)(128 / eb),
                             (cuuint32_t)(p.block_size < kTile ? p.block_size : kTile)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = f8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                    : (cache_dtype == MKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  CUtensorMap km, vm;
  CUresult r = enc(&km, dt, 2, const_cast<void*>(k_cache), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS)
    r = enc(&vm, dt, 2, const_cast<void*>(v_cache), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(MKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  if (p.num_units == 0) return MKV_OK;
  if (f8) {
    return q_dtype == MKV_DTYPE_BF16 ? launch_typed<bf16, fp8>(p, km, vm, stream, device)
                                     : launch_typed<f16, fp8>(p, km, vm, stream, device);
  }
  return q_dtype == MKV_DTYPE_BF16 ? launch_typed<bf16, bf16>(p, km, vm, stream, device)
                                   : launch_typed<f16, f16>(p, km, vm, stream, device);
}

}  // namespace tc05
}  // namespace mkv

#ifdef MKV_TC05_TRACE
extern "C" __attribute__((visibility("default"))) int mkv_debug_tc05_trace(unsigned long long* host, int n) {
  if (n > (int)sizeof(mkv::tc05::g_trace)) n = (int)sizeof(mkv::tc05::g_trace);
  return (int)cudaMemcpyFromSymbol(host, mkv::tc05::g_trace, n);
}
#endif
