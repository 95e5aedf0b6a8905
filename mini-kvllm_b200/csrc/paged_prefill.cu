// Chunked-prefill / extend attention over the paged KV cache.
//
// Reference behaviour (heart1128/mini-kvllm, src/myvllm/layers/attention.py):
//   paged_attention_prefill_kernel   attention.py:704-849  (wrapper 852-892, torch 649-701)
// Query token q of sequence b (q in [cu_seqlens_q[b], cu_seqlens_q[b+1])) at absolute
// position positions[q] attends to the cached tokens t < min(context_lens[b],
// positions[q] + 1), gathered through block_tables[b, t / block_size]; a -1 page is
// skipped; kv head of query head h is h / (H / KVH); out = softmax(scale q.K) V in fp32,
// stored in the query dtype. The reference has this path for unquantised caches only
// and lists the quantised one as a TODO (docs/chunked_prefill_todo.md:23-30); here the
// same kernel also reads e4m3 pages with a per-tensor scale and e4m3 / int8 pages with
// per-(page, row, kv head) scales, dequantised as the decode kernels do.
//
// B200 design (compute-bound once a chunk is long: ~4 * rows * ctx * D FLOP per
// (sequence, kv head), with K/V read once per kv head):
//   * a CTA owns 64 rows = (query token, query head of one kv head's group) pairs, so
//     the whole GQA group shares every K/V tile; query rows are staged once through
//     shared memory into ldmatrix A fragments;
//   * 64-token K/V tiles stream through a 2-stage cp.async ring (16-byte chunks,
//     XOR-swizzled per 8 rows); 8-bit pages are converted to the query dtype in shared
//     memory after they land (exact for e4m3 and int8);
//   * S = Q K^T and O += P V on the tensor cores (mma.sync m16n8k16, fp32 accumulate),
//     P reused from the S accumulators in registers (FlashAttention-2 form); per-row
//     causal visibility and -1 pages masked; online softmax in the exp2 domain with
//     quad shuffles;
//   * the (sequence, query block) of each CTA comes from a block scan of cu_seqlens_q,
//     so the host never reads device data (graph-safe).
// A CUDA-core kernel (one warp per query token and head) covers fp32 queries and head
// dims other than 64 / 128.
#include <cuda.h>
#include <cstdlib>

#include <cstdio>
#include <type_traits>

#include "mkv_common.cuh"
#include "sm100.cuh"

namespace mkv {
namespace {

constexpr int kPThreads = 128;
constexpr int kPRows = 64;   // (query token, head) rows per CTA
constexpr int kPKT = 64;     // kv tokens per tile

struct PrefillParams {
  const void* q;
  int64_t q_st, q_sh;  // elements
  const uint8_t* k_cache;
  const uint8_t* v_cache;
  int64_t num_blocks;
  int block_size;
  const void* bt;
  int64_t bt_sb;
  int max_blocks;
  int bt_i64;
  const void* ctx;
  int ctx_i64;
  const void* cu;
  int cu_i64;
  const void* pos;
  int pos_i64;
  int num_seqs, total_q, num_heads, num_kv_heads, head_dim, group;
  int qb;  // query tokens per CTA (kPRows / group)
  float qk_scale_log2;
  const float* k_scale;  // per-tensor scales of e4m3 pages, or null
  const float* v_scale;
  const float* k_scales;  // per-(page, row, kv head) scales of 8-bit pages, or null
  const float* v_scales;
  void* out;
  int64_t o_st, o_sh;  // elements
  // tcgen05 kernel over dequantised pages: page blk of sequence seq is scratch page
  // seq * max_blocks + blk of scratch_k / scratch_v (16-bit, the cache's row layout);
  // page validity still comes from the block table
  int scratch;
  const uint8_t* scratch_k;
  const uint8_t* scratch_v;
};

__device__ __forceinline__ int64_t ld_idx(const void* p, int i64, int64_t i) {
  return i64 ? (int64_t)__ldg(reinterpret_cast<const int64_t*>(p) + i)
             : (int64_t)__ldg(reinterpret_cast<const int32_t*>(p) + i);
}
__device__ __forceinline__ int64_t pf_cu(const PrefillParams& p, int64_t i) { return ld_idx(p.cu, p.cu_i64, i); }
__device__ __forceinline__ int64_t pf_pos(const PrefillParams& p, int64_t i) { return ld_idx(p.pos, p.pos_i64, i); }
__device__ __forceinline__ int64_t pf_ctx(const PrefillParams& p, int64_t i) { return ld_idx(p.ctx, p.ctx_i64, i); }

// Page of logical block blk of sequence seq, or -1 (entry -1 or out of range).
__device__ __forceinline__ int pf_page(const PrefillParams& p, int seq, int blk) {
  const int64_t idx = (int64_t)seq * p.bt_sb + blk;
  const int64_t page = p.bt_i64 ? (int64_t)__ldg((const int64_t*)p.bt + idx)
                                : (int64_t)__ldg((const int32_t*)p.bt + idx);
  return (page >= 0 && page < p.num_blocks) ? (int)page : -1;
}

// Tokens of the cache a query at position `pos` of a sequence with `ctx` cached tokens sees.
__device__ __forceinline__ int pf_visible(const PrefillParams& p, int64_t ctx, int64_t pos) {
  int64_t v = pos + 1 < ctx ? pos + 1 : ctx;
  const int64_t cap = (int64_t)p.max_blocks * p.block_size;
  if (v > cap) v = cap;
  return v > 0 ? (int)v : 0;
}

// (sequence, first query index, query tokens) of query block `unit`, units numbered
// sequence by sequence with ceil(len / qb) blocks each. Block-collective; false when
// `unit` is past the last block.
struct PfUnit {
  int seq, q0, nq;
};
template <int NTHREADS = kPThreads>
__device__ bool pf_find_unit(const PrefillParams& p, int64_t unit, PfUnit& u) {
  __shared__ long long red[NTHREADS / 32];
  __shared__ int found[3];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) found[0] = -1;
  long long carry = 0;
  for (int base = 0; base < p.num_seqs; base += NTHREADS) {
    const int s = base + tid;
    int len = 0;
    int64_t q0 = 0;
    if (s < p.num_seqs) {
      q0 = pf_cu(p, s);
      const int64_t q1 = pf_cu(p, s + 1);
      len = q1 > q0 ? (int)(q1 - q0) : 0;
    }
    const long long nb = (len + p.qb - 1) / p.qb;
    long long x = nb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long v = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += v;
    }
    __syncthreads();
    if (lane == 31) red[warp] = x;
    __syncthreads();
    long long off = carry, chunk = 0;
#pragma unroll
    for (int i = 0; i < NTHREADS / 32; ++i) {
      if (i < warp) off += red[i];
      chunk += red[i];
    }
    const long long incl = off + x;
    if (s < p.num_seqs && incl - nb <= unit && unit < incl) {
      const int b = (int)(unit - (incl - nb));
      found[0] = s;
      found[1] = (int)q0 + b * p.qb;
      found[2] = min(p.qb, len - b * p.qb);
    }
    carry += chunk;
    __syncthreads();
    if (carry > unit) break;
  }
  __syncthreads();
  u.seq = found[0];
  u.q0 = found[1];
  u.nq = found[2];
  return u.seq >= 0;
}

// ============================================================ tensor-core kernel
template <typename CT> struct PfByte { static constexpr bool kByte = false; };
template <> struct PfByte<fp8> { static constexpr bool kByte = true; };
template <> struct PfByte<int8_t> { static constexpr bool kByte = true; };

__device__ __forceinline__ float byte_to_f32(fp8 x) { return to_f32(x); }
__device__ __forceinline__ float byte_to_f32(int8_t x) { return (float)x; }

template <int D> struct PfLayout {
  static constexpr int ROWB = D * 2;                 // bytes per 16-bit row
  static constexpr int TILE = kPKT * ROWB;           // one 16-bit K or V tile
  static constexpr int QBYTES = kPRows * ROWB;       // query rows
};

// Shared memory: Q rows | 16-bit K/V tiles (2 stages, or 1 converted copy for 8-bit
// pages) | 8-bit staging (2 stages) | valid flags | per-token scales.
template <typename CT, int D>
constexpr size_t pf_smem_bytes() {
  using L = PfLayout<D>;
  constexpr bool kByte = PfByte<CT>::kByte;
  constexpr size_t tiles = (size_t)(kByte ? 1 : 2) * 2 * L::TILE;
  constexpr size_t raw = kByte ? (size_t)2 * 2 * kPKT * D : 0;
  return (size_t)L::QBYTES + tiles + raw + 2 * kPKT + (size_t)2 * 2 * kPKT * 4;
}

template <typename QT, typename CT, int D>
__global__ void __launch_bounds__(kPThreads, 1)
paged_prefill_tc_kernel(const PrefillParams p) {
  using L = PfLayout<D>;
  constexpr bool kByte = PfByte<CT>::kByte;
  constexpr int ROWB = L::ROWB;
  constexpr int CPR = ROWB / 16;  // 16-byte chunks per 16-bit row
  constexpr int RAWB = D * (int)sizeof(CT);
  constexpr int NT = D / 8;       // n-tiles of O
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* q_sm = smem;
  uint8_t* kv_sm = q_sm + L::QBYTES;                               // [stages][K, V] 16-bit
  uint8_t* raw_sm = kv_sm + (kByte ? 1 : 2) * 2 * L::TILE;         // [2][K, V] 8-bit
  uint8_t* valid = raw_sm + (kByte ? 2 * 2 * kPKT * D : 0);         // [2][kPKT]
  float* rsc = reinterpret_cast<float*>(valid + 2 * kPKT);          // [2][K, V][kPKT]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int kvh = blockIdx.y;
  PfUnit u;
  if (!pf_find_unit(p, blockIdx.x, u)) return;
  const int seq = u.seq;
  const int64_t ctx = pf_ctx(p, seq);
  const bool per_token = p.k_scales != nullptr;

  // ---- this thread's two rows (g and g + 8 of its warp): query index and visibility
  int vis[2];
  int qrow[2], hrow[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = warp * 16 + g + 8 * i;
    const int tok = r / p.group, gh = r - tok * p.group;
    const bool live = tok < u.nq;
    qrow[i] = live ? u.q0 + tok : -1;
    hrow[i] = kvh * p.group + gh;
    vis[i] = live ? pf_visible(p, ctx, pf_pos(p, u.q0 + tok)) : 0;
  }
  // kv tokens this CTA needs: the largest visibility of its rows
  __shared__ int vmax_s;
  if (tid == 0) vmax_s = 0;
  __syncthreads();
  atomicMax(&vmax_s, max(vis[0], vis[1]));
  // ---- stage the query rows (row r = token r / group, head r % group)
  const QT* qp = reinterpret_cast<const QT*>(p.q);
  for (int c = tid; c < kPRows * CPR; c += kPThreads) {
    const int r = c / CPR, k = c - r * CPR;
    const int tok = r / p.group, gh = r - tok * p.group;
    const bool live = tok < u.nq;
    const QT* src = qp + (int64_t)(u.q0 + (live ? tok : 0)) * p.q_st +
                    (int64_t)(kvh * p.group + gh) * p.q_sh + k * 8;
    cp_async_16(smem_u32(q_sm + r * ROWB + ((k ^ (r & 7)) << 4)), src, live ? 16 : 0);
  }
  cp_async_commit();
  __syncthreads();
  const int nkv = vmax_s;
  const int ntiles = (nkv + kPKT - 1) / kPKT;

  // ---- K/V tile loads: 16-byte chunks of the raw page rows
  const int64_t row_stride = (int64_t)p.num_kv_heads * RAWB;
  const int64_t head_off = (int64_t)kvh * RAWB;
  constexpr int RCPR = RAWB / 16;
  auto load_tile = [&](int it, int stage) {
    const int t0 = it * kPKT;
    uint8_t* kd = kByte ? raw_sm + stage * 2 * kPKT * RAWB : kv_sm + stage * 2 * L::TILE;
    uint8_t* vd = kd + (kByte ? kPKT * RAWB : L::TILE);
    for (int c = tid; c < kPKT * RCPR; c += kPThreads) {
      const int r = c / RCPR, k = c - r * RCPR;
      const int t = t0 + r;
      int page = -1, boff = 0;
      if (t < nkv) {
        const int blk = t / p.block_size;
        boff = t - blk * p.block_size;
        page = pf_page(p, seq, blk);
      }
      const bool ok = page >= 0;
      const int64_t off = ok ? ((int64_t)page * p.block_size + boff) * row_stride + head_off + k * 16 : 0;
      // 16-bit tiles are stored swizzled for ldmatrix; 8-bit staging is plain
      const int soff = kByte ? r * RAWB + k * 16 : r * ROWB + ((k ^ (r & 7)) << 4);
      cp_async_16(smem_u32(kd + soff), p.k_cache + off, ok ? 16 : 0);
      cp_async_16(smem_u32(vd + soff), p.v_cache + off, ok ? 16 : 0);
      if (k == 0) {
        valid[stage * kPKT + r] = ok ? 1 : 0;
        if (per_token) {
          const int64_t si = ok ? ((int64_t)page * p.block_size + boff) * p.num_kv_heads + kvh : 0;
          cp_async_4(smem_u32(rsc + stage * 2 * kPKT + r), p.k_scales + si, ok ? 4 : 0);
          cp_async_4(smem_u32(rsc + stage * 2 * kPKT + kPKT + r), p.v_scales + si, ok ? 4 : 0);
        }
      }
    }
  };
  if (ntiles > 0) load_tile(0, 0);
  cp_async_commit();

  // ---- Q fragments (A operand, rows x head_dim) from shared memory
  cp_async_wait<1>();  // the query group
  __syncthreads();
  const int lrow = lane & 7, lmat = lane >> 3;
  uint32_t qa[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int r = warp * 16 + ((lmat & 1) << 3) + lrow;
    const int ch = 2 * kk + (lmat >> 1);
    ldmatrix_x4(smem_u32(q_sm + r * ROWB + ((ch ^ (r & 7)) << 4)), qa[kk][0], qa[kk][1], qa[kk][2],
                qa[kk][3]);
  }
  const float ks_t = (kByte && !per_token) ? __ldg(p.k_scale) : 1.0f;
  const float vs_t = (kByte && !per_token) ? __ldg(p.v_scale) : 1.0f;
  const float sc = p.qk_scale_log2 * ks_t;

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};

  for (int it = 0; it < ntiles; ++it) {
    const int stage = it & 1;
    cp_async_wait<0>();
    __syncthreads();  // tile `it` is in; every warp is done with the previous tile
    if (it + 1 < ntiles) load_tile(it + 1, stage ^ 1);
    cp_async_commit();
    uint8_t* kt = kByte ? kv_sm : kv_sm + stage * 2 * L::TILE;
    uint8_t* vt = kt + L::TILE;
    if (kByte) {  // convert the 8-bit tile into the 16-bit (swizzled) tile
      const uint8_t* rk = raw_sm + stage * 2 * kPKT * RAWB;
      for (int c = tid; c < 2 * kPKT * (D / 8); c += kPThreads) {
        const int which = c / (kPKT * (D / 8));
        const int rem = c - which * kPKT * (D / 8);
        const int r = rem / (D / 8), k = rem - r * (D / 8);  // 8 elements = one 16-byte chunk out
        const uint2 raw = *reinterpret_cast<const uint2*>(rk + which * kPKT * RAWB + r * RAWB + k * 8);
        const CT* e = reinterpret_cast<const CT*>(&raw);
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = pack2<QT>(byte_to_f32(e[2 * j]), byte_to_f32(e[2 * j + 1]));
        *reinterpret_cast<uint4*>((which ? vt : kt) + r * ROWB + ((k ^ (r & 7)) << 4)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
      __syncthreads();
    }
    const uint8_t* vld = valid + stage * kPKT;
    const float* rk_s = rsc + stage * 2 * kPKT;

    // ---- S = Q K^T: 16 rows x 64 kv tokens per warp
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int r = jj * 16 + ((lmat >> 1) << 3) + lrow;
        const int ch = 2 * kk + (lmat & 1);
        uint32_t b[4];
        ldmatrix_x4(smem_u32(kt + r * ROWB + ((ch ^ (r & 7)) << 4)), b[0], b[1], b[2], b[3]);
        Mma<QT>::run(s[2 * jj], qa[kk], b[0], b[1]);
        Mma<QT>::run(s[2 * jj + 1], qa[kk], b[2], b[3]);
      }
    }

    // ---- mask, scale, online softmax (rows g and g + 8; a row's 4 threads are a quad)
    const int tbase = it * kPKT;
    float alpha[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = 8 * j + 2 * t4 + e;
          float x = s[j][2 * i + e] * sc;
          if (per_token) x *= rk_s[c];
          x = (tbase + c < vis[i] && vld[c]) ? x : -INFINITY;
          s[j][2 * i + e] = x;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[i], mx);
      const float base = m_new == -INFINITY ? 0.0f : m_new;
      alpha[i] = exp2f(m_run[i] - base);
      m_run[i] = m_new;
      float ls = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = exp2f(s[j][2 * i + e] - base);
          ls += pv;
          s[j][2 * i + e] = per_token ? pv * rk_s[kPKT + 8 * j + 2 * t4 + e] : pv;
        }
      l_run[i] = fmaf(l_run[i], alpha[i], ls);
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }

    // ---- O += P V: P from the S accumulators (A operand), V^T fragments by ldmatrix.trans
#pragma unroll
    for (int kk = 0; kk < kPKT / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack2<QT>(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack2<QT>(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack2<QT>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack2<QT>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int nd = 0; nd < D / 16; ++nd) {
        const int r = kk * 16 + ((lmat & 1) << 3) + lrow;
        const int ch = 2 * nd + (lmat >> 1);
        uint32_t b[4];
        ldmatrix_x4_trans(smem_u32(vt + r * ROWB + ((ch ^ (r & 7)) << 4)), b[0], b[1], b[2], b[3]);
        Mma<QT>::run(o[2 * nd], a, b[0], b[1]);
        Mma<QT>::run(o[2 * nd + 1], a, b[2], b[3]);
      }
    }
  }
  cp_async_wait<0>();

  // ---- normalise and store rows (query, head); 0/0 = NaN for a row that sees nothing
  QT* op = reinterpret_cast<QT*>(p.out);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float l = l_run[i];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (qrow[i] < 0) continue;
    const float inv = vs_t / l;
    QT* dst = op + (int64_t)qrow[i] * p.o_st + (int64_t)hrow[i] * p.o_sh;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int d = 8 * n + 2 * t4;
      *reinterpret_cast<uint32_t*>(dst + d) = pack2<QT>(o[n][2 * i] * inv, o[n][2 * i + 1] * inv);
    }
  }
}

// ============================================================ tcgen05 kernel
// 16-bit caches, head_dim 128, power-of-two block_size >= 8: a CTA owns NQ = 1 or 2 tiles
// of 128 rows (query token, GQA head) of one kv head and runs FlashAttention-2 with the
// accumulators and P in tensor memory:
//   warp 0     producer: 128-token K and V tiles by TMA (one 2D box per page segment and
//              64-column half, 128-byte swizzle) into separate K and V rings, K one tile
//              ahead of V (the order the MMAs consume them); a missing page's V rows are
//              zero-filled instead (its K columns are masked);
//   warp 1     MMA issuer: S = Q K(i)^T (M = N = 128, K = 128, operands K-major) into TMEM,
//              O += P V(i) with P read from TMEM (the first 64 columns of its S buffer, two
//              16-bit values per column) and V MN-major straight from the TMA tile. A K
//              stage is released when its last QK product completes, a V stage when its
//              last PV product does.
//              NQ = 1: two S buffers; QK(i) is issued one tile ahead of PV(i-1).
//              NQ = 2: one S buffer per query tile; PV_q(i) then QK_q(i+1), alternating
//              between the tiles, so that one tile's softmax runs while the other's
//              products do;
//   softmax    one warpgroup per query tile (warps 2-5, 6-9), thread = row = TMEM lane: S
//              row read once into registers, mask (causal per row, missing pages), online
//              softmax in the exp2 domain with a lazy reference (O in TMEM is rescaled
//              only when a row's maximum grows by more than 2^8), P stored into TMEM over
//              S; finally O / l to global memory.
// tcgen05.mma operations of a CTA run in issue order, so a QK product issued after PV(i)
// overwrites P(i) only after PV(i) has read it.
// Every mbarrier wait is bounded (sm100::kWaitCycles); a role that gives up raises the
// CTA abort flag, the others stop, in-flight TMA loads and MMAs are waited for (bounded)
// and TMEM is freed.
// 16 bytes of an 8-bit page row (CT = e4m3 or int8; byte i = element i) -> 16 values of
// QT in lo (elements 0-7) and hi (8-15). Conversions to half are exact; bf16 goes through
// fp32 (exact for e4m3 and int8 values). kTok: times the token's scale, in fp32 for bf16
// (one rounding) and in half for f16.
template <typename QT, typename CT, bool kTok>
__device__ __forceinline__ uint32_t pf_to_qt(uint32_t h, float scale) {
  if constexpr (!kTok && std::is_same<QT, f16>::value) {
    return h;
  } else if constexpr (kTok && std::is_same<QT, f16>::value) {
    const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&h), __float2half2_rn(scale));
    return *reinterpret_cast<const uint32_t*>(&r);
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
    return kTok ? pack2<QT>(f.x * scale, f.y * scale) : pack2<QT>(f.x, f.y);
  }
}
template <typename QT, typename CT, bool kTok>
__device__ __forceinline__ void pf_cvt16(const uint4 raw, float scale, uint4& lo, uint4& hi) {
  uint32_t h[8];
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if constexpr (std::is_same<CT, int8_t>::value) {
      h[2 * j] = s8x2_to_f16x2((uint16_t)w[j]);
      h[2 * j + 1] = s8x2_to_f16x2((uint16_t)(w[j] >> 16));
    } else {
      e4m3x4_to_f16x2x2(w[j], h[2 * j], h[2 * j + 1]);
    }
  }
  lo = make_uint4(pf_to_qt<QT, CT, kTok>(h[0], scale), pf_to_qt<QT, CT, kTok>(h[1], scale),
                  pf_to_qt<QT, CT, kTok>(h[2], scale), pf_to_qt<QT, CT, kTok>(h[3], scale));
  hi = make_uint4(pf_to_qt<QT, CT, kTok>(h[4], scale), pf_to_qt<QT, CT, kTok>(h[5], scale),
                  pf_to_qt<QT, CT, kTok>(h[6], scale), pf_to_qt<QT, CT, kTok>(h[7], scale));
}

namespace pf05 {
using namespace sm100;
constexpr int kRows = 128;     // MMA M: (query token, head) rows of one query tile
constexpr int kTile = 128;     // MMA N of S: kv tokens per tile
constexpr int kD = 128;
constexpr uint32_t kTmemCols = 512;  // S buffers (P over their first 64 columns) at 0 / 128, O at 256 (+128)
constexpr int BLK = 128 * 128;       // 128 rows x 128 bytes: one 64-column half
constexpr int TILE = 2 * BLK;        // 128 rows x 256 bytes
template <int NQ, bool kByte = false, bool kSplit = false>
struct Layout {
  // kSplit: one query tile, two softmax warpgroups, each taking half of S's columns
  static constexpr int kSoftmaxWarps = 4 * NQ * (kSplit ? 2 : 1);
  static constexpr int kConvWarps = kByte ? 4 : 0;  // 8-bit pages: converter warpgroup
  static constexpr int kThreads = 64 + 32 * kSoftmaxWarps + 32 * kConvWarps;
  static constexpr int kKStages = kByte ? 2 : 3;
  static constexpr int kVStages = kByte ? 2 : (NQ == 1 && !kSplit ? 3 : 2);
  static constexpr int kRStages = kByte ? 2 : 0;
  static constexpr int Q0 = 0;                           // [NQ] query tiles
  static constexpr int K0 = Q0 + NQ * TILE;              // [stage] K tile (16-bit)
  static constexpr int V0 = K0 + kKStages * TILE;        // [stage] V tile (16-bit)
  static constexpr int R0 = V0 + kVStages * TILE;        // [stage][K, V] 8-bit tiles, 128 x 128 B
  static constexpr int X0 = R0 + kRStages * 2 * BLK;     // kSplit: row maxima [2][2][128], sums [2][128]
  static constexpr int BAR0 = X0 + (kSplit ? 6 * kRows * 4 : 0);
  // K full/empty, V full/empty, raw full/empty, q, s[2], p[2], o[NQ], drain (+ x[2], l)
  static constexpr int NBAR = 2 * kKStages + 2 * kVStages + 2 * kRStages + 1 + 2 + 2 + NQ + 1 + (kSplit ? 3 : 0);
  static constexpr int MISC0 = BAR0 + NBAR * 8;          // tmem base, abort flag, nkv
  static constexpr int BYTES = MISC0 + 16 + 1024;        // + alignment slack
  static_assert(BYTES <= 232448, "shared memory per CTA");
  static_assert(!kByte || NQ == 1, "8-bit pages: one query tile (the converters take the other's warps)");
  static_assert(!kSplit || (NQ == 1 && !kByte), "split softmax: one query tile, 16-bit tiles");
};
}  // namespace pf05

template <typename QT, int NQ, typename CT, bool kTok, bool kSplit = false>
__global__ void __launch_bounds__(pf05::Layout<NQ, sizeof(CT) == 1, kSplit>::kThreads, 1)
paged_prefill_tc05_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap vmap, int units) {
  using namespace pf05;
  constexpr bool kByte = sizeof(CT) == 1;  // e4m3 or int8 pages, converted by warps 6-9
  using L = Layout<NQ, kByte, kSplit>;
  constexpr int kKS = L::kKStages, kVS = L::kVStages, kRS = L::kRStages;
  constexpr int kSoftmaxEnd = 2 + L::kSoftmaxWarps;  // softmax warps 2 .. kSoftmaxEnd - 1
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR0);
  uint64_t* kfull = bars;
  uint64_t* kempty = kfull + kKS;
  uint64_t* vfull = kempty + kKS;
  uint64_t* vempty = vfull + kVS;
  uint64_t* rfull = vempty + kVS;  // 8-bit tiles landed (TMA)
  uint64_t* rempty = rfull + kRS;  // 8-bit tiles converted
  uint64_t* qfull = rempty + kRS;
  uint64_t* sfull = qfull + 1;
  uint64_t* pfull = sfull + 2;
  uint64_t* ofull = pfull + 2;
  uint64_t* drain = ofull + NQ;
  uint64_t* xbar = drain + 1;  // kSplit: row-maximum exchange [2], row-sum exchange
  float* xch = reinterpret_cast<float*>(smem + L::X0);
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(smem + L::MISC0);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC0 + 4);
  int* nkv_s = reinterpret_cast<int*>(smem + L::MISC0 + 8);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.y;
  PfUnit u;
  // heaviest query blocks (latest in each sequence) first
  if (!pf_find_unit<L::kThreads>(p, (int64_t)units - 1 - blockIdx.x, u)) return;
  const int seq = u.seq;
  const int64_t ctx = pf_ctx(p, seq);

  if (tid == 0) {
    // 16-bit tiles are filled by TMA (one arrival + bytes); converted ones by the four
    // converter warps
    for (int s = 0; s < kKS; ++s) {
      mbar_init(&kfull[s], kByte ? 4 : 1);
      mbar_init(&kempty[s], 1);
    }
    for (int s = 0; s < kVS; ++s) {
      mbar_init(&vfull[s], kByte ? 4 : 1);
      mbar_init(&vempty[s], 1);
    }
    for (int s = 0; s < kRS; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 4);
    }
    mbar_init(qfull, L::kSoftmaxWarps);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfull[b], 1);
      mbar_init(&pfull[b], kSplit ? 8 : 4);
    }
    if (kSplit)
      for (int b = 0; b < 3; ++b) mbar_init(&xbar[b], 8);
    for (int q = 0; q < NQ; ++q) mbar_init(&ofull[q], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    *nkv_s = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_base_s, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_base_s;

  // softmax warp w in [2, kSoftmaxEnd) serves query tile qt = (w - 2) / 4; its thread owns
  // the tile's row rt = 32 * (w % 4) + lane, which is also its TMEM lane (warp w reaches
  // lanes 32 (w % 4) ..)
  const bool softmax_warp = warp >= 2 && warp < kSoftmaxEnd;
  // kSplit: warpgroup hh takes S columns 64 hh .. 64 hh + 63 of the one query tile
  const int hh = (kSplit && softmax_warp) ? (warp - 2) >> 2 : 0;
  const int qt = (softmax_warp && !kSplit) ? (warp - 2) >> 2 : 0;
  const int rt = 32 * (warp & 3) + lane;
  int vis = 0, qrow = -1, hrow = 0;
  if (softmax_warp) {
    const int row = kRows * qt + rt;
    const int tok = row / p.group, gh = row - tok * p.group;
    if (tok < u.nq) {
      qrow = u.q0 + tok;
      hrow = kvh * p.group + gh;
      vis = pf_visible(p, ctx, pf_pos(p, qrow));
    }
    atomicMax(nkv_s, vis);
  }
  __syncthreads();
  const int nkv = *nkv_s;
  const int ntiles = (nkv + kTile - 1) / kTile;
  // a tile is loaded in segments of one page (or of kTile tokens of a larger page)
  const int seg_rows = p.block_size < kTile ? p.block_size : kTile;
  const int nseg = kTile / seg_rows;

  if (warp == 0) {
    // ================================================================ producer
    if (lane == 0) {
      tma_prefetch_map(&kmap);
      tma_prefetch_map(&vmap);
    }
    // page of segment `lane` of tile t (-1: missing, or past the CTA's last kv token)
    auto seg_page_of = [&](int t) -> int {
      int pg = -1;
      if (lane < nseg) {
        const int ts = t * kTile + lane * seg_rows;
        if (ts < nkv) pg = pf_page(p, seq, ts / p.block_size);
      }
      return pg;
    };
    if constexpr (kByte) {
      // 8-bit pages: K(t) and V(t) together into one raw stage; missing segments are not
      // loaded (the converters write zeros for their rows)
      int nr = 0;  // raw stages issued
      bool ok = true;
      for (int t = 0; t < ntiles && ok; ++t) {
        if (__any_sync(0xffffffffu, *abort_flag != 0)) break;  // warp-uniform exit
        const int seg_page = seg_page_of(t);
        const int rs = t % kRS;
        ok = __all_sync(0xffffffffu, mbar_wait(&rempty[rs], ((t / kRS) & 1) ^ 1, abort_flag));
        if (!ok) break;
        uint32_t bytes = 0;
        for (int sgi = 0; sgi < nseg; ++sgi)
          if (__shfl_sync(0xffffffffu, seg_page, sgi) >= 0) bytes += 2u * seg_rows * 128u;
        if (lane == 0) mbar_arrive_expect_tx(&rfull[rs], bytes);
        uint8_t* dst = smem + L::R0 + rs * 2 * BLK;
        for (int sgi = 0; sgi < nseg; ++sgi) {
          const int pg = __shfl_sync(0xffffffffu, seg_page, sgi);
          if (lane == 0 && pg >= 0) {
            const int ts = t * kTile + sgi * seg_rows;
            const int y = pg * p.block_size + (ts & (p.block_size - 1));
            tma_load_2d(smem_u32(dst + sgi * seg_rows * 128), &kmap, kvh * kD, y, &rfull[rs]);
            tma_load_2d(smem_u32(dst + BLK + sgi * seg_rows * 128), &vmap, kvh * kD, y, &rfull[rs]);
          }
        }
        __syncwarp();
        ++nr;
      }
      if (!ok) *abort_flag = 1;
      if (lane == 0 && *abort_flag) {  // let issued loads land before the CTA exits
        for (int k = nr - kRS; k < nr; ++k)
          if (k >= 0) mbar_wait(&rfull[k % kRS], (k / kRS) & 1, nullptr);
      }
    } else {
      // K(t) and V(t) are issued in the order K(0), K(1), V(0), K(2), V(1), ...
      auto issue = [&](int t, bool is_v, int seg_page) -> bool {
        const int ns = is_v ? kVS : kKS;
        const int st = t % ns;
        uint64_t* empty = is_v ? vempty : kempty;
        uint64_t* full = is_v ? vfull : kfull;
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[st], ((t / ns) & 1) ^ 1, abort_flag))) return false;
        uint8_t* dst = smem + (is_v ? L::V0 : L::K0) + st * TILE;
        uint32_t bytes = 0;
        for (int sgi = 0; sgi < nseg; ++sgi) {
          const int pg = __shfl_sync(0xffffffffu, seg_page, sgi);
          if (pg >= 0) {
            bytes += 2u * seg_rows * 128u;
          } else if (is_v) {  // a missing segment's V rows: zeros (P is 0 there; 0 * garbage may not be)
            for (int k = lane; k < 2 * seg_rows * 8; k += 32) {
              const int b = k / (seg_rows * 8), kk = k - b * seg_rows * 8;
              *reinterpret_cast<uint4*>(dst + b * BLK + sgi * seg_rows * 128 + kk * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
          }
        }
        if (is_v) fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&full[st], bytes);
        for (int sgi = 0; sgi < nseg; ++sgi) {
          const int pg = __shfl_sync(0xffffffffu, seg_page, sgi);
          if (lane == 0 && pg >= 0) {
            const int ts = t * kTile + sgi * seg_rows;
            const int pg_row = p.scratch ? seq * p.max_blocks + ts / p.block_size : pg;
            const int y = pg_row * p.block_size + (ts & (p.block_size - 1));
            for (int b = 0; b < 2; ++b)
              tma_load_2d(smem_u32(dst + b * BLK + sgi * seg_rows * 128), is_v ? &vmap : &kmap,
                          kvh * kD + b * 64, y, &full[st]);
          }
        }
        __syncwarp();
        return true;
      };
      int nk = 0, nv = 0;  // K and V tiles issued
      int page_v = -1;     // segment pages of the V tile next in line
      bool ok = true;
      for (int t = 0; t <= ntiles && ok; ++t) {
        if (__any_sync(0xffffffffu, *abort_flag != 0)) break;  // warp-uniform exit
        const int page_k = t < ntiles ? seg_page_of(t) : -1;
        if (t < ntiles) {
          ok = issue(t, false, page_k);
          if (ok) ++nk;
        }
        if (ok && t > 0) {
          ok = issue(t - 1, true, page_v);
          if (ok) ++nv;
        }
        page_v = page_k;
      }
      if (!ok) *abort_flag = 1;
      if (lane == 0 && *abort_flag) {  // let issued loads land before the CTA exits
        for (int k = nk - kKS; k < nk; ++k)
          if (k >= 0) mbar_wait(&kfull[k % kKS], (k / kKS) & 1, nullptr);
        for (int k = nv - kVS; k < nv; ++k)
          if (k >= 0) mbar_wait(&vfull[k % kVS], (k / kVS) & 1, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ================================================================ MMA issuer
    constexpr uint32_t fmt = std::is_same<QT, bf16>::value ? 1u : 0u;
    constexpr uint32_t kIdQK = instr_desc(fmt, fmt, 0, 0, kRows, kTile);
    constexpr uint32_t kIdPV = instr_desc(fmt, fmt, 0, 1, kRows, kD);
    bool ok = ntiles == 0 || __all_sync(0xffffffffu, mbar_wait(qfull, 0, abort_flag));
    bool issued = false;  // any MMA issued (they must finish before TMEM is freed)
    // S_q(i) = Q_q K(i)^T into S buffer sb; release: the last QK product of K tile i
    auto qk = [&](int q, int i, int sb, bool release) -> bool {
      const int st = i % kKS;
      if (!__all_sync(0xffffffffu, mbar_wait(&kfull[st], (i / kKS) & 1, abort_flag))) return false;
      tc_fence_after_sync();
      if (lane == 0) {
        const uint32_t qaddr = smem_u32(smem + L::Q0 + q * TILE);
        const uint32_t kaddr = smem_u32(smem + L::K0 + st * TILE);
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {  // 16 head_dim columns per MMA
          const uint64_t a = smem_desc(qaddr + (k >> 2) * BLK + (k & 3) * 32, 16, 1024, kLayoutSw128);
          const uint64_t b = smem_desc(kaddr + (k >> 2) * BLK + (k & 3) * 32, 16, 1024, kLayoutSw128);
          mma_f16(tmem + sb * kTile, a, b, kIdQK, k > 0 ? 1u : 0u);
        }
        mma_commit(&sfull[sb]);
        if (release) mma_commit(&kempty[st]);
      }
      __syncwarp();
      issued = true;
      return true;
    };
    // O_q += P_q(j) V(j), P in S buffer sb (its pfull phase = ph); release: the last PV
    // product of V tile j
    auto pv = [&](int q, int j, int sb, int ph, bool release) -> bool {
      const int st = j % kVS;
      bool got = mbar_wait(&pfull[sb], ph, abort_flag) && mbar_wait(&vfull[st], (j / kVS) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, got)) return false;
      tc_fence_after_sync();
      if (lane == 0) {
        const uint32_t vaddr = smem_u32(smem + L::V0 + st * TILE);
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {  // 16 kv tokens per MMA = 8 TMEM columns of P
          const uint64_t b = smem_desc(vaddr + k * 2048, BLK, 1024, kLayoutSw128);
          // P of tokens 16k..: columns 8k (kSplit: the second half's P sits over its own S
          // at column 64 + 8(k - 4))
          const uint32_t pcol = sb * kTile + (kSplit && k >= 4 ? 32 + 8 * k : 8 * k);
          mma_f16_ts(tmem + 256 + q * kD, tmem + pcol, b, kIdPV, (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&ofull[q]);
        if (release) mma_commit(&vempty[st]);
      }
      __syncwarp();
      issued = true;
      return true;
    };
    if constexpr (NQ == 1) {
      for (int i = 0; i < ntiles && ok; ++i) {
        // S buffer i & 1 last held P(i-2), read by PV(i-2), which was issued before
        ok = qk(0, i, i & 1, true);
        if (ok && i > 0) ok = pv(0, i - 1, (i - 1) & 1, ((i - 1) >> 1) & 1, true);
      }
      if (ok && ntiles > 0) ok = pv(0, ntiles - 1, (ntiles - 1) & 1, ((ntiles - 1) >> 1) & 1, true);
    } else {
      // PV_q(i) then QK_q(i+1) (after PV_q(i), which reads P_q(i) from the S buffer
      // QK_q(i+1) overwrites), tile 0 then tile 1. (Polling both tiles' P barriers to take
      // whichever is ready first measured slower: the polling warp takes issue slots from
      // the softmax warps that share its SM sub-partition.)
      for (int q = 0; q < 2 && ok && ntiles > 0; ++q) ok = qk(q, 0, q, q == 1);
      for (int i = 0; i < ntiles && ok; ++i) {
        for (int q = 0; q < 2 && ok; ++q) {
          ok = pv(q, i, q, i & 1, q == 1);
          if (ok && i + 1 < ntiles) ok = qk(q, i + 1, q, q == 1);
        }
      }
    }
    if (!ok) *abort_flag = 1;
    if (lane == 0 && issued) {  // every MMA of this CTA done before TMEM is freed
      mma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
    __syncwarp();
  } else if (softmax_warp) {
    // ================================================================ softmax (warpgroup qt)
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t o_col = 256 + qt * kD;
    // stage this row of Q (128-byte swizzle, two 64-column halves)
    {
      const QT* src = reinterpret_cast<const QT*>(p.q) + (int64_t)(qrow >= 0 ? qrow : 0) * p.q_st +
                      (int64_t)hrow * p.q_sh;
      uint8_t* qdst = smem + L::Q0 + qt * TILE + rt * 128;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        if (kSplit && (c >> 3) != hh) continue;  // each warpgroup stages its half of the row
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (qrow >= 0) v = *reinterpret_cast<const uint4*>(src + c * 8);
        const int b = c >> 3, cc = c & 7;
        *reinterpret_cast<uint4*>(qdst + b * BLK + ((cc ^ (rt & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(qfull);
    }
    // per-tensor scales of 8-bit pages fold into the score scale and the output; per-(token,
    // head) scales were applied by the converters
    const bool tensor_scales = p.k_scale != nullptr;  // set only with per-tensor 8-bit pages
    const float sc = p.qk_scale_log2 * (tensor_scales ? __ldg(p.k_scale) : 1.0f);
    const float out_scale = tensor_scales ? __ldg(p.v_scale) : 1.0f;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    // page of segment `lane` of tile t (0 past the CTA's last kv token), looked up one
    // tile ahead
    auto seg_page_of = [&](int t) -> int {
      const int ts = t * kTile + lane * seg_rows;
      return (lane < nseg && ts < nkv) ? pf_page(p, seq, ts / p.block_size) : 0;
    };
    int pg_next = ntiles > 0 ? seg_page_of(0) : 0;
    for (int i = 0; i < ntiles && ok; ++i) {
      const int sb = NQ == 1 ? (i & 1) : qt;
      const int ph = NQ == 1 ? ((i >> 1) & 1) : (i & 1);
      const int t0 = i * kTile;
      const int pg = pg_next;
      if (i + 1 < ntiles) pg_next = seg_page_of(i + 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&sfull[sb], ph, abort_flag));
      if (!ok) break;
      const uint32_t bad = __ballot_sync(0xffffffffu, pg < 0);  // bit s: segment s missing
      tc_fence_after_sync();
      const uint32_t sa = tmem + lane_base + sb * kTile;
      // mask: the causal edge of this row (tokens >= vis, which also covers tokens past
      // the context) and missing pages
      uint32_t mw[4];
      bool all = true;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int r = vis - t0 - 32 * k;
        mw[k] = r >= 32 ? 0xffffffffu : (r <= 0 ? 0u : (1u << r) - 1u);
      }
      if (bad != 0u) {
#pragma unroll 1
        for (int sgi = 0; sgi < nseg; ++sgi) {
          if (!((bad >> sgi) & 1u)) continue;
          const int t = sgi * seg_rows;  // segment's first token in the tile
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (seg_rows >= 32) {
              if (32 * k >= t && 32 * k < t + seg_rows) mw[k] = 0u;
            } else if (k == (t >> 5)) {
              mw[k] &= ~(((1u << seg_rows) - 1u) << (t & 31));
            }
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) all = all && mw[k] == 0xffffffffu;
      all = all || qrow < 0;  // padding rows are never written
      const bool masked = !__all_sync(0xffffffffu, all);
      auto apply_mask = [&](float* v, int c0, int n) {
        if (masked) {
#pragma unroll
          for (int e = 0; e < n; ++e)
            if (!((mw[(c0 + e) >> 5] >> ((c0 + e) & 31)) & 1u)) v[e] = -INFINITY;
        }
      };
      // P = 2^(s sc - ref) of columns 64h .. 64h + 63 as 16-bit pairs into w, their sum into
      // acc and their raw maximum into mx8
      auto p_half = [&](int h, float ref, uint32_t (&w)[32], uint64_t (&acc)[4], float (&mx8)[8]) {
        float v[64];
        tmem_ld64(sa + 64 * h, v);
        apply_mask(v, 64 * h, 64);
#pragma unroll
        for (int e = 0; e < 64; e += 16)
#pragma unroll
          for (int k = 0; k < 8; ++k) mx8[k] = fmax3(mx8[k], v[e + k], v[e + 8 + k]);
        const uint64_t sc2 = f2_pack(sc, sc), nref2 = f2_pack(-ref, -ref);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(v[2 * e], v[2 * e + 1]), sc2, nref2), x0, x1);
          const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);  // 0 for masked (-inf)
          acc[e & 3] = f2_add(acc[e & 3], f2_pack(p0, p1));
          w[e] = pack2<QT>(p0, p1);
        }
      };
      // both halves: P into w0 / w1; returns the row sum, the raw row maximum into mxr
      auto p_tile = [&](float ref, uint32_t (&w0)[32], uint32_t (&w1)[32], float& mxr) -> float {
        uint64_t acc[4];
        float mx8[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[k] = f2_pack(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
        if constexpr (kSplit) {
          p_half(hh, ref, w0, acc, mx8);  // this warpgroup's half only
        } else {
          p_half(0, ref, w0, acc, mx8);
          reg_fence32(w0);
          p_half(1, ref, w1, acc, mx8);
        }
        mxr = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float a0, a1;
          f2_unpack(acc[k], a0, a1);
          sum += a0 + a1;
        }
        return sum;
      };
      // One pass in the common case: P against the current reference m, computed together
      // with the tile's maximum, is kept unless a row's maximum grew by more than 2^8 (the
      // lazy rescale threshold); then, and on a row's first visible tile, P is computed again
      // against the new maximum. S stays in TMEM until P is stored.
      uint32_t w0[32], w1[32];
      float lsum, mxr;
      bool need;
      float m_new, alpha;
      // kSplit: the row maximum of the two halves, exchanged through shared memory
      // (buffer and barrier alternate by tile; bounded wait)
      auto combine_max = [&]() -> bool {
        if constexpr (kSplit) {
          float* x = xch + (i & 1) * 2 * kRows;
          x[hh * kRows + rt] = mxr;
          __syncwarp();
          if (lane == 0) mbar_arrive(&xbar[i & 1]);
          if (!__all_sync(0xffffffffu, mbar_wait(&xbar[i & 1], (i >> 1) & 1, abort_flag))) return false;
          mxr = fmaxf(x[rt], x[kRows + rt]);
        }
        return true;
      };
      // lazy reference: move it (and rescale O) only when the maximum grows by > 2^8
      auto new_ref = [&]() {
        const float mx = mxr * sc;  // the scale is > 0
        need = mx > m + 8.0f;
        m_new = need ? mx : m;
        alpha = need ? exp2f(m - m_new) : 1.0f;  // 0 when m was -inf
      };
      if (__any_sync(0xffffffffu, m == -INFINITY)) {
        // a row's first visible tile: the maximum first (64 columns at a time)
        float mx8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          if (kSplit && h != hh) continue;
          float v[64];
          tmem_ld64(sa + 64 * h, v);
          apply_mask(v, 64 * h, 64);
#pragma unroll
          for (int e = 0; e < 64; e += 16)
#pragma unroll
            for (int k = 0; k < 8; ++k) mx8[k] = fmax3(mx8[k], v[e + k], v[e + 8 + k]);
        }
        mxr = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        if (!combine_max()) {
          ok = false;
          break;
        }
        new_ref();
        float unused;
        lsum = p_tile(m_new == -INFINITY ? 0.0f : m_new, w0, w1, unused);
      } else {
        lsum = p_tile(m, w0, w1, mxr);
        if (!combine_max()) {
          ok = false;
          break;
        }
        new_ref();
        if (__any_sync(0xffffffffu, need)) {
          float unused;
          lsum = p_tile(m_new, w0, w1, unused);
        }
      }
      m = m_new;
      l = l * alpha + lsum;
      // P over the first 64 columns of this S buffer (kSplit: each half's P over the first
      // 32 columns of its own S half)
      if constexpr (kSplit) {
        tmem_st32(sa + 64 * hh, w0);
      } else {
        tmem_st32(sa, w0);
        tmem_st32(sa + 32, w1);
      }
      // PV(i-1) done: O may be rescaled, and the next wait on this O barrier is for PV(i)
      if (i > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&ofull[qt], (i - 1) & 1, abort_flag));
        if (!ok) break;
        tc_fence_after_sync();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = kSplit ? 4 * hh : 0; c < (kSplit ? 4 * hh + 4 : kD / 16); ++c) {
            float v[16];
            tmem_ld16(tmem + lane_base + o_col + 16 * c, v);
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] *= alpha;
            tmem_st16(tmem + lane_base + o_col + 16 * c, v);
          }
        }
      }
      tmem_wait_st();
      // V rows past the last visible token of every row may hold anything (the page's
      // other tokens or never-written memory): zero them so that 0 * V stays 0. Query
      // tile 0 does it, before its PV product, which is issued before tile 1's.
      if (!kByte && qt == 0 && hh == 0 && t0 + kTile > nkv) {
        const int st = i % kVS;
        ok = __all_sync(0xffffffffu, mbar_wait(&vfull[st], (i / kVS) & 1, abort_flag));
        if (!ok) break;
        if (t0 + rt >= nkv) {
          uint8_t* vrow = smem + L::V0 + st * TILE + rt * 128;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            *reinterpret_cast<uint4*>(vrow + k * 16) = make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(vrow + BLK + k * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        fence_proxy_async_smem();
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[sb]);
    }
    if (!ok) *abort_flag = 1;
    // ---- epilogue: out = O / l (0/0 = NaN for a row that sees nothing)
    if (ok && ntiles > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&ofull[qt], (ntiles - 1) & 1, abort_flag));
      if (!ok) *abort_flag = 1;
      tc_fence_after_sync();
    }
    if constexpr (kSplit) {  // the row sum is split between the halves too
      float* xl = xch + 4 * kRows;
      xl[hh * kRows + rt] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[2]);
      if (!__all_sync(0xffffffffu, mbar_wait(&xbar[2], 0, abort_flag))) {
        ok = false;
        *abort_flag = 1;
      }
      l = xl[rt] + xl[kRows + rt];
    }
    const float inv = out_scale / l;
    QT* dst = reinterpret_cast<QT*>(p.out) + (int64_t)(qrow >= 0 ? qrow : 0) * p.o_st + (int64_t)hrow * p.o_sh;
#pragma unroll 1
    for (int c = kSplit ? 4 * hh : 0; c < (kSplit ? 4 * hh + 4 : kD / 16); ++c) {
      float v[16];
      if (ntiles > 0 && ok) {
        tmem_ld16(tmem + lane_base + o_col + 16 * c, v);
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0.0f;
      }
      if (qrow >= 0) {
        uint32_t w[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) w[e >> 1] = pack2<QT>(v[e] * inv, v[e + 1] * inv);
        *reinterpret_cast<uint4*>(dst + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(dst + 16 * c + 8) = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
  } else if constexpr (kByte) {
    // ================================================================ converters (warps 6-9)
    // Thread r converts row r (kv token t0 + r) of each K and V tile from the raw 8-bit
    // stage (128-byte swizzle) into the 16-bit tiles the MMAs read, multiplying by the
    // token's scales in the per-(token, head) modes. Rows of missing pages and rows past
    // the CTA's last kv token become zeros (P is 0 there, and 0 * V must stay 0).
    const int r = 32 * (warp - kSoftmaxEnd) + lane;
    auto page_of = [&](int t) -> int {
      const int tok = t * kTile + r;
      return tok < nkv ? pf_page(p, seq, tok / p.block_size) : -1;
    };
    auto convert_row = [&](const uint8_t* src_tile, uint8_t* dst_tile, bool valid, float scale) {
      uint8_t* drow = dst_tile + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
        if (valid) {
          const uint4 raw = *reinterpret_cast<const uint4*>(src_tile + r * 128 + ((c ^ (r & 7)) << 4));
          pf_cvt16<QT, CT, kTok>(raw, scale, lo, hi);
        }
        const int b = c >> 2, cc = (c & 3) * 2;  // columns 16c .. -> half b, chunks cc, cc + 1
        *reinterpret_cast<uint4*>(drow + b * BLK + ((cc ^ (r & 7)) << 4)) = lo;
        *reinterpret_cast<uint4*>(drow + b * BLK + (((cc + 1) ^ (r & 7)) << 4)) = hi;
      }
    };
    // the row's page is looked up two tiles ahead and its scales one tile ahead
    auto scales_of = [&](int t, int pg, float& ks, float& vs) {
      ks = vs = 1.0f;
      if (kTok && pg >= 0) {
        const int64_t slot = (int64_t)pg * p.block_size + ((t * kTile + r) & (p.block_size - 1));
        ks = __ldg(p.k_scales + slot * p.num_kv_heads + kvh);
        vs = __ldg(p.v_scales + slot * p.num_kv_heads + kvh);
      }
    };
    bool ok = true;
    int pg_cur = ntiles > 0 ? page_of(0) : -1;
    int pg_nxt = ntiles > 1 ? page_of(1) : -1;
    float ks_nxt, vs_nxt;
    scales_of(0, pg_cur, ks_nxt, vs_nxt);
    for (int i = 0; i < ntiles && ok; ++i) {
      const int rs = i % kRS, st = i % kKS;  // kKS == kVS
      const int pg = pg_cur;
      const float ks = ks_nxt, vs = vs_nxt;
      pg_cur = pg_nxt;
      if (i + 2 < ntiles) pg_nxt = page_of(i + 2);
      if (i + 1 < ntiles) scales_of(i + 1, pg_cur, ks_nxt, vs_nxt);
      ok = mbar_wait(&rfull[rs], (i / kRS) & 1, abort_flag) &&
           mbar_wait(&kempty[st], ((i / kKS) & 1) ^ 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      const uint8_t* raw = smem + L::R0 + rs * 2 * BLK;
      convert_row(raw, smem + L::K0 + st * TILE, pg >= 0, ks);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&kfull[st]);
      ok = __all_sync(0xffffffffu, mbar_wait(&vempty[st], ((i / kVS) & 1) ^ 1, abort_flag));
      if (!ok) break;
      convert_row(raw + BLK, smem + L::V0 + st * TILE, pg >= 0, vs);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&vfull[st]);
        mbar_arrive(&rempty[rs]);
      }
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

typedef CUresult (*PfEncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PfEncodeTiledFn pf_encode_fn() {  // resolved once (thread-safe static initialisation)
  static const PfEncodeTiledFn fn = []() -> PfEncodeTiledFn {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PfEncodeTiledFn>(f);
    return nullptr;
  }();
  return fn;
}

// tcgen05 path: head_dim 128, GQA group <= 128, power-of-two block size >= 8, 16-byte
// aligned output rows, 16-bit queries; the cache in the query dtype, or e4m3 (per-tensor
// or per-(token, head) scales), or int8 (per-(token, head) scales).
bool pf05_supported(const PrefillParams& p, int q_dtype, int cache_dtype) {
  if (p.head_dim != pf05::kD || p.group > pf05::kRows || !(p.qk_scale_log2 > 0.0f)) return false;
  if (q_dtype != MKV_DTYPE_BF16 && q_dtype != MKV_DTYPE_F16) return false;
  const bool same = cache_dtype == q_dtype;
  const bool fp8 = cache_dtype == MKV_DTYPE_FP8_E4M3 && (p.k_scale != nullptr || p.k_scales != nullptr);
  const bool int8 = cache_dtype == MKV_DTYPE_INT8 && p.k_scales != nullptr;
  if (!same && !fp8 && !int8) return false;
  if (p.block_size < 8 || (p.block_size & (p.block_size - 1)) != 0) return false;
  if (((uintptr_t)p.out & 15u) || (p.o_st * 2) % 16 != 0 || (p.o_sh * 2) % 16 != 0) return false;
  return pf_encode_fn() != nullptr;
}

template <typename QT, int NQ, typename CT, bool kTok = false, bool kSplit = false>
int launch_prefill_tc05(const PrefillParams& p, int cache_dtype, cudaStream_t stream) {
  constexpr bool kByte = sizeof(CT) == 1;
  using L = pf05::Layout<NQ, kByte, kSplit>;
  PfEncodeTiledFn enc = pf_encode_fn();
  // rows of the cache = (page, offset) slots; a row holds KVH heads of head_dim elements.
  // 16-bit tiles are loaded as two 64-column halves, 8-bit tiles as one 128-byte box.
  const int64_t map_pages = p.scratch ? (int64_t)p.num_seqs * p.max_blocks : p.num_blocks;
  const uint8_t* kbase = p.scratch ? p.scratch_k : p.k_cache;
  const uint8_t* vbase = p.scratch ? p.scratch_v : p.v_cache;
  const cuuint64_t dims[2] = {(cuuint64_t)p.num_kv_heads * pf05::kD,
                              (cuuint64_t)map_pages * (cuuint64_t)p.block_size};
  const cuuint64_t strides[1] = {(cuuint64_t)p.num_kv_heads * pf05::kD * sizeof(CT)};
  const cuuint32_t box[2] = {kByte ? 128u : 64u,
                             (cuuint32_t)(p.block_size < pf05::kTile ? p.block_size : pf05::kTile)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = kByte ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                       : (cache_dtype == MKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  CUtensorMap km, vm;
  CUresult r = enc(&km, dt, 2, const_cast<uint8_t*>(kbase), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS)
    r = enc(&vm, dt, 2, const_cast<uint8_t*>(vbase), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  {  // the shared-memory opt-in, once per kernel and CUDA context
    const int st = ensure_dynamic_smem((const void*)paged_prefill_tc05_kernel<QT, NQ, CT, kTok, kSplit>,
                                       (int)L::BYTES, "cudaFuncSetAttribute(prefill tc05 smem)");
    if (st != MKV_OK) return st;
  }
  PrefillParams q = p;
  q.qb = NQ * pf05::kRows / p.group;  // query tokens per CTA: 128 NQ rows
  const int64_t units = (int64_t)q.total_q / q.qb + q.num_seqs;
  dim3 grid((unsigned)units, q.num_kv_heads, 1);
  paged_prefill_tc05_kernel<QT, NQ, CT, kTok, kSplit><<<grid, L::kThreads, L::BYTES, stream>>>(q, km, vm, (int)units);
  return cuda_status(cudaGetLastError(), "paged_prefill_tc05 launch");
}

// Two query tiles per CTA keep the tensor core busy while a tile's softmax runs, but
// leave more rows idle when sequences contribute few rows. They are used when the
// average sequence holds at least two CTAs' worth of rows and the grid still fills the
// GPU twice over. 8-bit caches always use one (their converter warps take the other
// tile's share of the register file).
// MKV_PREFILL_QTILES=1 or 2 in the environment overrides the choice for 16-bit caches
// (tests, tuning).
template <typename QT>
int launch_prefill_tc05_auto(const PrefillParams& p, int cache_dtype, cudaStream_t stream) {
  if (cache_dtype == MKV_DTYPE_FP8_E4M3)
    return p.k_scales != nullptr ? launch_prefill_tc05<QT, 1, fp8, true>(p, cache_dtype, stream)
                                 : launch_prefill_tc05<QT, 1, fp8, false>(p, cache_dtype, stream);
  if (cache_dtype == MKV_DTYPE_INT8) return launch_prefill_tc05<QT, 1, int8_t, true>(p, cache_dtype, stream);
  const char* force = getenv("MKV_PREFILL_QTILES");
  if (force != nullptr && force[0] == '1') return launch_prefill_tc05<QT, 1, QT, false, true>(p, cache_dtype, stream);
  if (force != nullptr && force[0] == '2') return launch_prefill_tc05<QT, 2, QT>(p, cache_dtype, stream);
  const int64_t rows = (int64_t)p.total_q * p.group;
  const int64_t ctas2 = (rows + 2 * pf05::kRows - 1) / (2 * pf05::kRows) * p.num_kv_heads;
  if (rows >= (int64_t)p.num_seqs * 4 * pf05::kRows && ctas2 >= 2 * kNumSMs)
    return launch_prefill_tc05<QT, 2, QT>(p, cache_dtype, stream);
  return launch_prefill_tc05<QT, 1, QT, false, true>(p, cache_dtype, stream);
}

// ============================================================ 8-bit pages -> 16-bit scratch
// For long chunks the tcgen05 kernel reads 16-bit copies of the 8-bit pages, made once
// per call, instead of converting every tile again in each of the many CTAs that share a
// sequence and kv head. Page blk of sequence seq (its tokens below context_lens[seq]) is
// converted into scratch page seq * max_blocks + blk, with the cache's row layout
// (block_size rows of KVH x 128 values); per-(token, head) scales are applied here, and
// per-tensor scales stay with the attention kernel. Missing pages are skipped: the
// attention kernel masks their tokens and zero-fills their V rows.
template <typename QT, typename CT, bool kTok>
__global__ void __launch_bounds__(256) prefill_dequant_pages_kernel(const PrefillParams p, QT* sk, QT* sv) {
  const int blk = blockIdx.x, seq = blockIdx.y;
  const int64_t ctx = pf_ctx(p, seq);
  const int64_t t0 = (int64_t)blk * p.block_size;
  if (t0 >= ctx) return;
  const int page = pf_page(p, seq, blk);
  if (page < 0) return;
  constexpr int kChunks = pf05::kD / 16;  // 16-byte raw chunks per (token, head)
  const int per_tok = p.num_kv_heads * kChunks;
  const int ntok = (int)(ctx - t0 < p.block_size ? ctx - t0 : p.block_size);
  const int64_t row_elems = (int64_t)p.num_kv_heads * pf05::kD;
  const int64_t src_row0 = (int64_t)page * p.block_size;
  const int64_t dst_row0 = ((int64_t)seq * p.max_blocks + blk) * p.block_size;
  for (int c = threadIdx.x; c < ntok * per_tok; c += blockDim.x) {
    const int tok = c / per_tok, hc = c - tok * per_tok;  // hc = head * kChunks + chunk
    const int64_t src = (src_row0 + tok) * row_elems + hc * 16;
    const int64_t dst = (dst_row0 + tok) * row_elems + hc * 16;
    float ks = 1.0f, vs = 1.0f;
    if constexpr (kTok) {
      const int64_t si = (src_row0 + tok) * p.num_kv_heads + hc / kChunks;
      ks = __ldg(p.k_scales + si);
      vs = __ldg(p.v_scales + si);
    }
    uint4 lo, hi;
    pf_cvt16<QT, CT, kTok>(__ldg(reinterpret_cast<const uint4*>(p.k_cache + src)), ks, lo, hi);
    *reinterpret_cast<uint4*>(sk + dst) = lo;
    *reinterpret_cast<uint4*>(sk + dst + 8) = hi;
    pf_cvt16<QT, CT, kTok>(__ldg(reinterpret_cast<const uint4*>(p.v_cache + src)), vs, lo, hi);
    *reinterpret_cast<uint4*>(sv + dst) = lo;
    *reinterpret_cast<uint4*>(sv + dst + 8) = hi;
  }
}

constexpr size_t kScratchCap = (size_t)1 << 30;  // largest scratch the library asks for

// Bytes of the 16-bit page scratch for a call, or 0 when the converter kernel is used:
// 8-bit cache, 16-bit queries, head_dim 128, GQA group <= 128, power-of-two block size
// >= 8, sequences with at least 512 query rows (query tokens x GQA group) on average, and
// at most kScratchCap.
size_t prefill_scratch_bytes(int32_t num_seqs, int64_t total_q, int32_t num_heads,
                             int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                             int32_t max_num_blocks, int32_t q_dtype, int32_t cache_dtype) {
  if (cache_dtype != MKV_DTYPE_FP8_E4M3 && cache_dtype != MKV_DTYPE_INT8) return 0;
  if (q_dtype != MKV_DTYPE_BF16 && q_dtype != MKV_DTYPE_F16) return 0;
  if (head_dim != pf05::kD || num_seqs <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return 0;
  const int64_t group = num_heads / num_kv_heads;
  if (group > pf05::kRows || block_size < 8 || (block_size & (block_size - 1)) != 0) return 0;
  if (max_num_blocks <= 0 || total_q * group < (int64_t)num_seqs * 4 * pf05::kRows) return 0;
  const double bytes = 2.0 * num_seqs * (double)max_num_blocks * block_size * num_kv_heads * head_dim * 2.0;
  if (bytes > (double)kScratchCap) return 0;
  return (size_t)bytes;
}

template <typename QT, typename CT, bool kTok>
int launch_prefill_scratch(const PrefillParams& p, int q_dtype, void* workspace, cudaStream_t s) {
  const size_t half = (size_t)p.num_seqs * p.max_blocks * p.block_size * p.num_kv_heads * pf05::kD;
  QT* sk = reinterpret_cast<QT*>(workspace);
  QT* sv = sk + half;
  dim3 grid((unsigned)p.max_blocks, (unsigned)p.num_seqs, 1);
  prefill_dequant_pages_kernel<QT, CT, kTok><<<grid, 256, 0, s>>>(p, sk, sv);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "prefill_dequant_pages launch");
  PrefillParams q = p;
  q.scratch = 1;
  q.scratch_k = reinterpret_cast<const uint8_t*>(sk);
  q.scratch_v = reinterpret_cast<const uint8_t*>(sv);
  q.k_scales = q.v_scales = nullptr;  // per-token scales were applied by the conversion
  return launch_prefill_tc05_auto<QT>(q, q_dtype, s);
}

// ============================================================ CUDA-core kernel
// One warp per (query token, query head): lanes take 32 cached tokens at a time, the
// warp keeps the online softmax state, and each lane accumulates head_dim / 32 outputs.
template <typename QT, typename CT>
__global__ void __launch_bounds__(kPThreads)
paged_prefill_generic_kernel(const PrefillParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int D = p.head_dim;
  const bool byte_pages = sizeof(CT) == 1;
  const bool per_token = p.k_scales != nullptr;
  const float ks_t = (byte_pages && !per_token) ? __ldg(p.k_scale) : 1.0f;
  const float vs_t = (byte_pages && !per_token) ? __ldg(p.v_scale) : 1.0f;
  const CT* kc = reinterpret_cast<const CT*>(p.k_cache);
  const CT* vc = reinterpret_cast<const CT*>(p.v_cache);
  const QT* qp = reinterpret_cast<const QT*>(p.q);
  QT* op = reinterpret_cast<QT*>(p.out);
  constexpr int kMaxPer = 8;  // head_dim <= 256
  for (int64_t w = wid; w < (int64_t)p.total_q * p.num_heads; w += nwarps) {
    const int64_t q = w / p.num_heads;
    const int h = (int)(w - q * p.num_heads);
    const int kvh = h / p.group;
    // sequence of query q: the last b with cu[b] <= q (binary search)
    int lo = 0, hi = p.num_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pf_cu(p, mid) <= q) lo = mid; else hi = mid - 1;
    }
    const int seq = lo;
    if (q >= pf_cu(p, seq + 1)) continue;  // not inside any sequence (malformed cu): skip
    const int nvis = pf_visible(p, pf_ctx(p, seq), pf_pos(p, q));
    float qv[kMaxPer], acc[kMaxPer];
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int d = lane + 32 * j;
      qv[j] = d < D ? to_f32(qp[q * p.q_st + (int64_t)h * p.q_sh + d]) * p.qk_scale_log2 * ks_t : 0.0f;
      acc[j] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    for (int t0 = 0; t0 < nvis; t0 += 32) {
      const int t = t0 + lane;
      float sco = -INFINITY, vsc = 0.0f;
      int64_t row = -1;
      if (t < nvis) {
        const int blk = t / p.block_size;
        const int page = pf_page(p, seq, blk);
        if (page >= 0)
          row = ((int64_t)page * p.block_size + (t - blk * p.block_size)) * p.num_kv_heads + kvh;
      }
      // scores: lanes with a token compute q . k with q broadcast from its owner lane
      float dot = 0.0f;
      for (int d = 0; d < D; ++d) {
        const float qd = __shfl_sync(0xffffffffu, qv[d >> 5], d & 31);
        if (row >= 0) dot = fmaf(qd, to_f32(kc[row * D + d]), dot);
      }
      if (row >= 0) {
        sco = dot;
        if (per_token) {
          sco *= __ldg(p.k_scales + row);
          vsc = __ldg(p.v_scales + row);
        } else {
          vsc = 1.0f;
        }
      }
      float mx = sco;
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
      const float m_new = fmaxf(m, mx);
      const float base = m_new == -INFINITY ? 0.0f : m_new;
      const float alpha = exp2f(m - base);
      const float pv = exp2f(sco - base);  // 0 for lanes without a token
      float ps = pv;
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o2);
      l = l * alpha + ps;
      m = m_new;
#pragma unroll
      for (int j = 0; j < kMaxPer; ++j) acc[j] *= alpha;
      const float wv = pv * vsc;
      for (int src = 0; src < 32; ++src) {
        const float wj = __shfl_sync(0xffffffffu, wv, src);
        const int64_t rj = __shfl_sync(0xffffffffu, row, src);
        if (rj < 0) continue;
#pragma unroll
        for (int j = 0; j < kMaxPer; ++j) {
          const int d = lane + 32 * j;
          if (d < D) acc[j] = fmaf(wj, to_f32(vc[rj * D + d]), acc[j]);
        }
      }
    }
    const float inv = vs_t / l;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int d = lane + 32 * j;
      if (d < D) op[q * p.o_st + (int64_t)h * p.o_sh + d] = from_f32<QT>(acc[j] * inv);
    }
  }
}

template <typename QT, typename CT, int D>
int launch_prefill_tc(const PrefillParams& p, int64_t units, cudaStream_t stream) {
  constexpr size_t smem = pf_smem_bytes<CT, D>();
  {  // the shared-memory opt-in, once per kernel and CUDA context
    const int st = ensure_dynamic_smem((const void*)paged_prefill_tc_kernel<QT, CT, D>, (int)smem,
                                       "cudaFuncSetAttribute(prefill smem)");
    if (st != MKV_OK) return st;
  }
  dim3 grid((unsigned)units, p.num_kv_heads, 1);
  paged_prefill_tc_kernel<QT, CT, D><<<grid, kPThreads, smem, stream>>>(p);
  return cuda_status(cudaGetLastError(), "paged_prefill_tc launch");
}

template <typename QT, typename CT>
int launch_prefill_generic(const PrefillParams& p, cudaStream_t stream) {
  int64_t warps = (int64_t)p.total_q * p.num_heads;
  int64_t blocks = (warps + kPThreads / 32 - 1) / (kPThreads / 32);
  if (blocks > (int64_t)kNumSMs * 16) blocks = (int64_t)kNumSMs * 16;
  if (blocks < 1) blocks = 1;
  paged_prefill_generic_kernel<QT, CT><<<(unsigned)blocks, kPThreads, 0, stream>>>(p);
  return cuda_status(cudaGetLastError(), "paged_prefill_generic launch");
}

template <typename QT>
int dispatch_prefill(const PrefillParams& p, int cache_dtype, int64_t units, cudaStream_t s,
                     int q_dtype, void* ws, size_t ws_bytes) {
  if constexpr (!std::is_same<QT, float>::value) {
    if (pf05_supported(p, q_dtype, cache_dtype)) {
      const size_t need = prefill_scratch_bytes(p.num_seqs, p.total_q, p.num_heads, p.num_kv_heads,
                                                p.head_dim, p.block_size, p.max_blocks, q_dtype,
                                                cache_dtype);
      if (need > 0 && ws != nullptr && ws_bytes >= need && ((uintptr_t)ws & 15u) == 0) {
        if (cache_dtype == MKV_DTYPE_FP8_E4M3)
          return p.k_scales != nullptr ? launch_prefill_scratch<QT, fp8, true>(p, q_dtype, ws, s)
                                       : launch_prefill_scratch<QT, fp8, false>(p, q_dtype, ws, s);
        return launch_prefill_scratch<QT, int8_t, true>(p, q_dtype, ws, s);
      }
      return launch_prefill_tc05_auto<QT>(p, cache_dtype, s);
    }
    if ((p.head_dim == 128 || p.head_dim == 64) && p.group <= kPRows) {
      if (cache_dtype == MKV_DTYPE_FP8_E4M3)
        return p.head_dim == 128 ? launch_prefill_tc<QT, fp8, 128>(p, units, s)
                                 : launch_prefill_tc<QT, fp8, 64>(p, units, s);
      if (cache_dtype == MKV_DTYPE_INT8)
        return p.head_dim == 128 ? launch_prefill_tc<QT, int8_t, 128>(p, units, s)
                                 : launch_prefill_tc<QT, int8_t, 64>(p, units, s);
      return p.head_dim == 128 ? launch_prefill_tc<QT, QT, 128>(p, units, s)
                               : launch_prefill_tc<QT, QT, 64>(p, units, s);
    }
  }
  if (cache_dtype == MKV_DTYPE_FP8_E4M3) return launch_prefill_generic<QT, fp8>(p, s);
  if (cache_dtype == MKV_DTYPE_INT8) return launch_prefill_generic<QT, int8_t>(p, s);
  return launch_prefill_generic<QT, QT>(p, s);
}

}  // namespace
}  // namespace mkv

// ============================================================ contiguous (varlen) prefill
// Causal attention of each sequence over its own contiguous K/V rows, the reference's
// flash_attention_prefill (attention.py:446-516, kernel 336-443), which Attention.forward
// takes for a batch of whole prompts (context.is_full_prefill, attention.py:1771) and the
// runner's warm-up takes before any KV cache exists (model_runner.py:193-200).
// B200 design: the rows are packed once into 128-row pages of a caller workspace (sequence
// b owns pages [page_start[b], page_start[b] + ceil(len_b / 128)), page_start an exclusive
// scan of the page counts), with a block table, lengths and positions built on the
// device; the tcgen05 paged prefill then runs over those pages unchanged (query row q of
// sequence b at position t sees tokens 0..t). The pack is one read and one write of K/V,
// small beside the quadratic attention; the host never reads device data.
namespace mkv {
namespace {
constexpr int kVarlenPage = 128;

template <typename I>
__device__ __forceinline__ int64_t ld_cu(const void* cu, int i) {
  return (int64_t)reinterpret_cast<const I*>(cu)[i];
}
__device__ __forceinline__ int64_t cu_at(const void* cu, int cu_i64, int i) {
  return cu_i64 ? ld_cu<int64_t>(cu, i) : ld_cu<int32_t>(cu, i);
}

// One CTA: page starts (exclusive scan of ceil(len / 128) in chunks of the block), block
// tables (num_seqs x max_pages, -1 padded) and lengths.
__global__ void __launch_bounds__(1024)
varlen_tables_kernel(const void* cu, int cu_i64, int num_seqs, int max_pages, int* page_start,
                     int* bt, int* lens) {
  __shared__ int warp_sum[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int carry = 0;
  for (int base = 0; base < num_seqs; base += blockDim.x) {
    const int b = base + threadIdx.x;
    int len = 0;
    if (b < num_seqs) {
      const int64_t l = cu_at(cu, cu_i64, b + 1) - cu_at(cu, cu_i64, b);
      len = l > 0 ? (int)l : 0;
    }
    const int np = (len + kVarlenPage - 1) / kVarlenPage;
    int x = np;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += v;
    }
    if (lane == 31) warp_sum[warp] = x;
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < nwarps; ++w) {
      if (w < warp) before += warp_sum[w];
      total += warp_sum[w];
    }
    const int start = carry + before + x - np;
    if (b < num_seqs) {
      page_start[b] = start;
      lens[b] = len;
      int* row = bt + (int64_t)b * max_pages;
      for (int j = 0; j < max_pages; ++j) row[j] = j < np ? start + j : -1;
    }
    carry += total;
    __syncthreads();  // warp_sum is rewritten by the next chunk
  }
}

// One thread per 16-byte chunk of a (token, kv head) row of K and of V: token i of
// sequence b (binary search of cu_seqlens) at position t = i - cu[b] goes to row
// page_start[b] * 128 + t of the pages; positions[i] = t.
__global__ void __launch_bounds__(256)
varlen_pack_kernel(const uint8_t* __restrict__ k, const uint8_t* __restrict__ v, int64_t k_st,
                   int64_t k_sh, int64_t v_st, int64_t v_sh,  // bytes
                   const void* cu, int cu_i64, int num_seqs, int64_t total, int num_kv_heads,
                   int chunks, const int* __restrict__ page_start, uint8_t* __restrict__ pk,
                   uint8_t* __restrict__ pv, int* __restrict__ positions) {
  const int64_t per_token = (int64_t)num_kv_heads * chunks;
  const int64_t items = total * per_token;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < items;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = idx / per_token;
    const int rem = (int)(idx - i * per_token);
    const int h = rem / chunks, c = rem - h * chunks;
    int lo = 0, hi = num_seqs;  // largest b with cu[b] <= i
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (cu_at(cu, cu_i64, mid) <= i) lo = mid; else hi = mid;
    }
    const int64_t t = i - cu_at(cu, cu_i64, lo);
    const int64_t row = (int64_t)page_start[lo] * kVarlenPage + t;
    const int64_t dst = (row * num_kv_heads + h) * (int64_t)chunks * 16 + c * 16;
    st_v4(pk + dst, ld_stream_v4(k + i * k_st + h * k_sh + c * 16));
    st_v4(pv + dst, ld_stream_v4(v + i * v_st + h * v_sh + c * 16));
    if (h == 0 && c == 0) positions[i] = (int)t;
  }
}

struct VarlenLayout {
  int64_t pages;
  size_t pk, pv, bt, lens, pos, start, total;
};
VarlenLayout varlen_layout(int num_seqs, int64_t total, int max_seqlen, int num_kv_heads,
                           int head_dim, int eb) {
  VarlenLayout L{};
  const int max_pages = (max_seqlen + kVarlenPage - 1) / kVarlenPage;
  L.pages = (total + kVarlenPage - 1) / kVarlenPage + num_seqs;
  const size_t page_bytes = (size_t)kVarlenPage * num_kv_heads * head_dim * eb;
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  L.pk = 0;
  L.pv = up(L.pages * page_bytes);
  L.bt = L.pv + up(L.pages * page_bytes);
  L.lens = L.bt + up((size_t)num_seqs * max_pages * 4);
  L.pos = L.lens + up((size_t)num_seqs * 4);
  L.start = L.pos + up((size_t)total * 4);
  L.total = L.start + up((size_t)num_seqs * 4);
  return L;
}
}  // namespace
}  // namespace mkv

using namespace mkv;

extern "C" int mkv_paged_prefill(
    const void* query, int64_t q_stride_token, int64_t q_stride_head, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t cache_dtype, const float* k_scale,
    const float* v_scale, const float* k_scales, const float* v_scales, int64_t num_blocks,
    int32_t block_size, const void* block_tables, int32_t block_table_index_type,
    int64_t block_table_stride_seq, int32_t max_num_blocks, const void* context_lens,
    int32_t context_lens_index_type, const void* cu_seqlens_q, int32_t cu_seqlens_index_type,
    const void* positions, int32_t positions_index_type, int32_t num_seqs, int64_t total_q,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float scale, void* out,
    int64_t out_stride_token, int64_t out_stride_head, void* workspace, size_t workspace_bytes,
    void* stream) {
  clear_error();
  const char* fn = "mkv_paged_prefill";
  if (num_seqs < 0 || total_q < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_size <= 0 || max_num_blocks < 0 || num_blocks < 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: bad sizes", fn);
  if (num_heads % num_kv_heads != 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "%s: num_heads (%d) must be a multiple of num_kv_heads (%d)", fn, num_heads,
                     num_kv_heads);
  for (int t : {block_table_index_type, context_lens_index_type, cu_seqlens_index_type,
                positions_index_type})
    if (t != MKV_INDEX_I32 && t != MKV_INDEX_I64)
      return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: bad index type", fn);
  if (num_seqs == 0 || total_q == 0) return MKV_OK;
  if (!query || !k_cache || !v_cache || !context_lens || !cu_seqlens_q || !positions || !out ||
      (max_num_blocks > 0 && !block_tables))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (total_q > (int64_t)1 << 31 || (int64_t)max_num_blocks * block_size >= ((int64_t)1 << 31))
    return set_error(MKV_ERR_UNSUPPORTED, "%s: sizes beyond 2^31", fn);
  if (head_dim % 16 != 0 || head_dim > 256)
    return set_error(MKV_ERR_UNSUPPORTED,
                     "%s: head_dim must be a multiple of 16 and at most 256 (got %d)", fn, head_dim);
  if (q_dtype != MKV_DTYPE_F32 && q_dtype != MKV_DTYPE_F16 && q_dtype != MKV_DTYPE_BF16)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: query dtype must be f32, f16 or bf16", fn);
  const bool byte_cache = cache_dtype == MKV_DTYPE_FP8_E4M3 || cache_dtype == MKV_DTYPE_INT8;
  const bool per_token = k_scales != nullptr || v_scales != nullptr;
  if (per_token && (!k_scales || !v_scales))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: both k_scales and v_scales are needed", fn);
  if (!byte_cache && cache_dtype != q_dtype)
    return set_error(MKV_ERR_UNSUPPORTED,
                     "%s: cache dtype (%d) must equal the query dtype (%d) for float caches", fn,
                     cache_dtype, q_dtype);
  if (byte_cache && !per_token && (cache_dtype == MKV_DTYPE_INT8 || !k_scale || !v_scale))
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "%s: an 8-bit cache needs per-tensor scales (FP8) or per-token scales", fn);
  if (per_token && !byte_cache)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: per-token scales need an 8-bit cache", fn);
  if (((uintptr_t)k_cache & 15u) || ((uintptr_t)v_cache & 15u))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: caches must be 16-byte aligned", fn);
  const int64_t qeb = q_dtype == MKV_DTYPE_F32 ? 4 : 2;
  const int group = num_heads / num_kv_heads;
  const bool tc_shape = (head_dim == 128 || head_dim == 64) && q_dtype != MKV_DTYPE_F32 &&
                        group <= kPRows;
  if (tc_shape && (((uintptr_t)query & 15u) || (q_stride_token * qeb) % 16 != 0 ||
                   (q_stride_head * qeb) % 16 != 0 || ((uintptr_t)out & 3u) ||
                   (out_stride_token * qeb) % 4 != 0 || (out_stride_head * qeb) % 4 != 0))
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "%s: query rows must be 16-byte aligned and output rows 4-byte aligned", fn);
  PrefillParams p;
  p.q = query;
  p.q_st = q_stride_token;
  p.q_sh = q_stride_head;
  p.k_cache = (const uint8_t*)k_cache;
  p.v_cache = (const uint8_t*)v_cache;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.bt = block_tables;
  p.bt_sb = block_table_stride_seq;
  p.max_blocks = max_num_blocks;
  p.bt_i64 = block_table_index_type == MKV_INDEX_I64;
  p.ctx = context_lens;
  p.ctx_i64 = context_lens_index_type == MKV_INDEX_I64;
  p.cu = cu_seqlens_q;
  p.cu_i64 = cu_seqlens_index_type == MKV_INDEX_I64;
  p.pos = positions;
  p.pos_i64 = positions_index_type == MKV_INDEX_I64;
  p.num_seqs = num_seqs;
  p.total_q = (int)total_q;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.group = group;
  p.qb = group <= kPRows ? kPRows / group : 1;
  p.qk_scale_log2 = scale * 1.4426950408889634f;
  p.k_scale = byte_cache && !per_token ? k_scale : nullptr;
  p.v_scale = byte_cache && !per_token ? v_scale : nullptr;
  p.k_scales = per_token ? k_scales : nullptr;
  p.v_scales = per_token ? v_scales : nullptr;
  p.out = out;
  p.o_st = out_stride_token;
  p.o_sh = out_stride_head;
  p.scratch = 0;
  p.scratch_k = p.scratch_v = nullptr;
  // query blocks: at most one partial block per sequence beyond total_q / qb full ones
  const int64_t units = total_q / p.qb + num_seqs;
  cudaStream_t s = (cudaStream_t)stream;
  switch (q_dtype) {
    case MKV_DTYPE_F32: return dispatch_prefill<float>(p, cache_dtype, units, s, q_dtype, workspace, workspace_bytes);
    case MKV_DTYPE_F16: return dispatch_prefill<f16>(p, cache_dtype, units, s, q_dtype, workspace, workspace_bytes);
    default: return dispatch_prefill<bf16>(p, cache_dtype, units, s, q_dtype, workspace, workspace_bytes);
  }
}

extern "C" size_t mkv_paged_prefill_workspace_bytes(
    int32_t num_seqs, int64_t total_q, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
    int32_t block_size, int32_t max_num_blocks, int32_t q_dtype, int32_t cache_dtype) {
  return prefill_scratch_bytes(num_seqs, total_q, num_heads, num_kv_heads, head_dim, block_size,
                               max_num_blocks, q_dtype, cache_dtype);
}


extern "C" size_t mkv_varlen_prefill_workspace_bytes(int32_t num_seqs, int64_t total_tokens,
                                                     int32_t max_seqlen, int32_t num_kv_heads,
                                                     int32_t head_dim, int32_t dtype) {
  if (num_seqs <= 0 || total_tokens <= 0 || max_seqlen <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return 0;
  const int eb = dtype == MKV_DTYPE_F32 ? 4 : 2;
  return varlen_layout(num_seqs, total_tokens, max_seqlen, num_kv_heads, head_dim, eb).total;
}

extern "C" int mkv_varlen_prefill(
    const void* query, int64_t q_stride_token, int64_t q_stride_head, int32_t dtype,
    const void* key, const void* value, int64_t key_stride_token, int64_t key_stride_head,
    int64_t value_stride_token, int64_t value_stride_head, const void* cu_seqlens,
    int32_t cu_seqlens_index_type, int32_t num_seqs, int64_t total_tokens, int32_t max_seqlen,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float scale, void* out,
    int64_t out_stride_token, int64_t out_stride_head, void* workspace, size_t workspace_bytes,
    void* stream) {
  clear_error();
  const char* fn = "mkv_varlen_prefill";
  if (num_seqs < 0 || total_tokens < 0 || max_seqlen < 0 || num_heads <= 0 || num_kv_heads <= 0 ||
      head_dim <= 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: bad sizes", fn);
  if (cu_seqlens_index_type != MKV_INDEX_I32 && cu_seqlens_index_type != MKV_INDEX_I64)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: bad cu_seqlens index type", fn);
  if (dtype != MKV_DTYPE_F32 && dtype != MKV_DTYPE_F16 && dtype != MKV_DTYPE_BF16)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: dtype must be f32, f16 or bf16", fn);
  if (num_seqs == 0 || total_tokens == 0) return MKV_OK;
  if (!query || !key || !value || !cu_seqlens || !out || !workspace)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (max_seqlen <= 0 || max_seqlen > total_tokens)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: max_seqlen must be in [1, total_tokens]", fn);
  if (total_tokens >= ((int64_t)1 << 31))
    return set_error(MKV_ERR_UNSUPPORTED, "%s: total_tokens must be < 2^31", fn);
  const int eb = dtype == MKV_DTYPE_F32 ? 4 : 2;
  const int64_t row_bytes = (int64_t)head_dim * eb;
  if (row_bytes % 16 != 0 || ((uintptr_t)key & 15u) || ((uintptr_t)value & 15u) ||
      (key_stride_token * eb) % 16 || (key_stride_head * eb) % 16 ||
      (value_stride_token * eb) % 16 || (value_stride_head * eb) % 16)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: key/value rows must be 16-byte aligned", fn);
  const VarlenLayout L = varlen_layout(num_seqs, total_tokens, max_seqlen, num_kv_heads, head_dim, eb);
  if (workspace_bytes < L.total || ((uintptr_t)workspace & 255u))
    return set_error(MKV_ERR_WORKSPACE, "%s: workspace of %zu bytes (256-byte aligned) needed, %zu given",
                     fn, L.total, workspace_bytes);
  const int max_pages = (max_seqlen + kVarlenPage - 1) / kVarlenPage;
  uint8_t* ws = (uint8_t*)workspace;
  int* bt = (int*)(ws + L.bt);
  int* lens = (int*)(ws + L.lens);
  int* pos = (int*)(ws + L.pos);
  int* start = (int*)(ws + L.start);
  cudaStream_t s = (cudaStream_t)stream;
  const int cu_i64 = cu_seqlens_index_type == MKV_INDEX_I64;
  varlen_tables_kernel<<<1, 1024, 0, s>>>(cu_seqlens, cu_i64, num_seqs, max_pages, start, bt, lens);
  int st = cuda_status(cudaGetLastError(), "varlen_tables launch");
  if (st != MKV_OK) return st;
  const int chunks = (int)(row_bytes / 16);
  const int64_t items = total_tokens * num_kv_heads * chunks;
  int64_t blocks = (items + 255) / 256;
  if (blocks > (int64_t)kNumSMs * 16) blocks = (int64_t)kNumSMs * 16;
  varlen_pack_kernel<<<(unsigned)blocks, 256, 0, s>>>(
      (const uint8_t*)key, (const uint8_t*)value, key_stride_token * eb, key_stride_head * eb,
      value_stride_token * eb, value_stride_head * eb, cu_seqlens, cu_i64, num_seqs, total_tokens,
      num_kv_heads, chunks, start, ws + L.pk, ws + L.pv, pos);
  st = cuda_status(cudaGetLastError(), "varlen_pack launch");
  if (st != MKV_OK) return st;
  st = mkv_paged_prefill(query, q_stride_token, q_stride_head, dtype, ws + L.pk, ws + L.pv, dtype,
                         nullptr, nullptr, nullptr, nullptr, L.pages, kVarlenPage, bt, MKV_INDEX_I32,
                         max_pages, max_pages, lens, MKV_INDEX_I32, cu_seqlens, cu_seqlens_index_type,
                         pos, MKV_INDEX_I32, num_seqs, total_tokens, num_heads, num_kv_heads,
                         head_dim, scale, out, out_stride_token, out_stride_head, nullptr, 0, stream);
  if (st != MKV_OK) {  // name this entry point in the message
    char msg[512];
    snprintf(msg, sizeof(msg), "%s", mkv_last_error());
    return set_error(st, "%s: %s", fn, msg);
  }
  return MKV_OK;
}
