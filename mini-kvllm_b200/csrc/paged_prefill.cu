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
#include <cstdio>
#include <type_traits>

#include "mkv_common.cuh"

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
__device__ bool pf_find_unit(const PrefillParams& p, int64_t unit, PfUnit& u) {
  __shared__ long long red[kPThreads / 32];
  __shared__ int found[3];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) found[0] = -1;
  long long carry = 0;
  for (int base = 0; base < p.num_seqs; base += kPThreads) {
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
    for (int i = 0; i < kPThreads / 32; ++i) {
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
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(paged_prefill_tc_kernel<QT, CT, D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(prefill smem)");
    configured[dev] = true;
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
int dispatch_prefill(const PrefillParams& p, int cache_dtype, int64_t units, cudaStream_t s) {
  if constexpr (!std::is_same<QT, float>::value) {
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
    int64_t out_stride_token, int64_t out_stride_head, void* stream) {
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
  // query blocks: at most one partial block per sequence beyond total_q / qb full ones
  const int64_t units = total_q / p.qb + num_seqs;
  cudaStream_t s = (cudaStream_t)stream;
  switch (q_dtype) {
    case MKV_DTYPE_F32: return dispatch_prefill<float>(p, cache_dtype, units, s);
    case MKV_DTYPE_F16: return dispatch_prefill<f16>(p, cache_dtype, units, s);
    default: return dispatch_prefill<bf16>(p, cache_dtype, units, s);
  }
}
