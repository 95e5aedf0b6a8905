// Paged-attention decode: one query token per sequence against its paged K/V.
//
// Reference behaviour (heart1128/mini-kvllm, src/myvllm/layers/attention.py):
//   paged_attention_decode_kernel      attention.py:517-646  (bf16/fp16/fp32 cache)
//   paged_attention_decode_fp8_kernel  attention.py:953-1121 (PER_TOKEN_HEAD=0: per-tensor scales)
//   wrappers                           attention.py:895-950, 1213-1268
// Semantics kept: kv_head = h / (H / KVH); tokens t < context_len whose logical block
// t / block_size is < max_num_blocks; page = block_tables[b, t / block_size] with -1
// meaning "skip this token"; FP8 values dequantised as float(e4m3) * scale; output
// = softmax(scale * q.K) V in fp32, stored in the query dtype.
//
// B200 design (HBM-bound: ~2 * G FLOP per cache byte):
//   * one CTA per (sequence, kv head, KV split) covers the whole GQA group, so each
//     page row is read from HBM once, not G times as in the reference's (seq, head) grid;
//   * pages stream through a multi-stage cp.async ring of 64-token tiles in shared
//     memory (16-byte chunks, XOR-swizzled so ldmatrix reads are conflict-free);
//   * QK^T and PV run on the tensor cores (mma.sync m16n8k16, fp32 accumulate) with
//     the query group as the M=16 rows; FP8 pages are converted e4m3x2 -> f16x2 in
//     registers straight out of ldmatrix, so dequantisation adds no memory traffic;
//     the per-tensor K scale is folded into the score scale and V's into the output;
//   * online softmax in the exp2 domain with quad shuffles; 4 warps split each tile
//     and merge their (m, l, acc) through shared memory at the end;
//   * long or ragged contexts are split into fixed-size token chunks (flash-decoding)
//     and merged by a second kernel; a sequence that fits one chunk writes its output
//     directly. The split count depends only on shapes, so the launch is graph-safe.
// A CUDA-core kernel with the same tiling covers fp32 and other head dims.
#include <type_traits>

#include "mkv_common.cuh"

namespace mkv {
namespace {

constexpr int kThreads = 128;      // 4 warps per CTA (both kernels)
constexpr int kMaxHeadsPerCta = 16;  // query heads of one KV head handled by a CTA
constexpr int kTcTile = 64;        // tokens per pipeline stage, tensor-core kernel
constexpr int kGenTile = 32;       // tokens per pipeline stage, CUDA-core kernel
constexpr int kChunkAlign = 64;    // split boundaries are multiples of both tiles
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  const void* q;
  int64_t q_sb, q_sh;  // elements
  const uint8_t* k_cache;
  const uint8_t* v_cache;
  int64_t num_blocks;
  int block_size;
  int bs_shift;  // log2(block_size) when it is a power of two, else -1
  const void* bt;
  int64_t bt_sb;
  int max_blocks;
  int bt_i64;
  const void* ctx;
  int ctx_i64;
  int num_seqs, num_heads, num_kv_heads, head_dim;
  int group;          // H / KVH
  int heads_per_cta;  // min(group, kMaxHeadsPerCta)
  int head_groups;    // ceil(group / heads_per_cta)
  float qk_scale_log2;  // attention scale * log2(e)
  const float* k_scale;  // FP8 per-tensor scales (nullptr for float caches)
  const float* v_scale;
  void* out;
  int64_t o_sb, o_sh;  // elements
  float* part_acc;  // [num_seqs][num_heads][num_splits][head_dim]
  float* part_ml;   // [num_seqs][num_heads][num_splits][2] = (m in log2 units, l)
  int num_splits;
  int chunk;  // tokens per split, multiple of kChunkAlign
  int32_t* invalid;
};

__device__ __forceinline__ int64_t load_ctx(const DecodeParams& p, int seq) {
  return p.ctx_i64 ? (int64_t)__ldg((const int64_t*)p.ctx + seq)
                   : (int64_t)__ldg((const int32_t*)p.ctx + seq);
}

// Page of logical token t of sequence seq, or -1 when the token has no valid page.
// Entries outside [0, num_blocks) other than -1 are counted once per (seq, token).
__device__ __forceinline__ int64_t page_of_block(const DecodeParams& p, int seq, int blk,
                                                 bool count) {
  const int64_t idx = (int64_t)seq * p.bt_sb + blk;
  const int64_t page = p.bt_i64 ? (int64_t)__ldg((const int64_t*)p.bt + idx)
                                : (int64_t)__ldg((const int32_t*)p.bt + idx);
  if (page >= 0 && page < p.num_blocks) return page;
  if (page != -1 && count && p.invalid != nullptr) atomicAdd(p.invalid, 1);
  return -1;
}

// (logical block, row in block) of token t; contexts are < 2^31 tokens (host-checked).
__device__ __forceinline__ void split_token(const DecodeParams& p, int t, int& blk, int& off) {
  if (p.bs_shift >= 0) {
    blk = t >> p.bs_shift;
    off = t & ((1 << p.bs_shift) - 1);
  } else {
    blk = t / p.block_size;
    off = t - blk * p.block_size;
  }
}

// Token range of this CTA's split and the number of splits the sequence uses.
struct SplitRange {
  int64_t begin, end;
  int active;
};
__device__ __forceinline__ SplitRange split_range(const DecodeParams& p, int seq, int split) {
  int64_t ctx = load_ctx(p, seq);
  const int64_t cap = (int64_t)p.max_blocks * p.block_size;
  int64_t eff = ctx < cap ? ctx : cap;
  if (eff < 0) eff = 0;
  SplitRange r;
  r.active = eff > 0 ? (int)((eff + p.chunk - 1) / p.chunk) : 1;
  r.begin = (int64_t)split * p.chunk;
  r.end = r.begin + p.chunk < eff ? r.begin + p.chunk : eff;
  return r;
}

// ============================================================ CUDA-core kernel
// Any float cache type, runtime head_dim (multiple of 16, <= 256). A warp scores one
// head over the 32 tokens of a tile (lane = token), the softmax update runs per head
// with warp shuffles, and PV gives each thread head_dim/128 output columns.
template <typename QT, typename CT>
__global__ void __launch_bounds__(kThreads)
paged_decode_generic_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int EB = sizeof(CT);
  constexpr bool kFp8 = std::is_same<CT, fp8>::value;
  constexpr int kPer = 16 / EB;  // elements per 16-byte chunk
  const int D = p.head_dim;
  const int row_bytes = D * EB;
  const int row_pitch = row_bytes + 16;  // padding keeps lane-per-row reads conflict-free
  const int chunks = row_bytes / 16;

  uint8_t* kbuf = smem;                                   // [2][kGenTile][row_pitch]
  uint8_t* vbuf = kbuf + 2 * kGenTile * row_pitch;         // [2][kGenTile][row_pitch]
  float* q_s = reinterpret_cast<float*>(vbuf + 2 * kGenTile * row_pitch);  // [16][D]
  float* s_s = q_s + kMaxHeadsPerCta * D;                 // [16][kGenTile]
  float* m_s = s_s + kMaxHeadsPerCta * kGenTile;          // [16]
  float* l_s = m_s + kMaxHeadsPerCta;                     // [16]
  float* a_s = l_s + kMaxHeadsPerCta;                     // [16]
  uint8_t* valid = reinterpret_cast<uint8_t*>(a_s + kMaxHeadsPerCta);  // [2][kGenTile]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.head_groups;
  const int hg = blockIdx.y - kvh * p.head_groups;
  const int seq = blockIdx.z;
  const int h0 = kvh * p.group + hg * p.heads_per_cta;
  const int nh = min(p.heads_per_cta, p.group - hg * p.heads_per_cta);
  const bool count_invalid = (kvh == 0 && hg == 0);

  const SplitRange rng = split_range(p, seq, split);
  if (split > 0 && rng.begin >= rng.end) return;

  const float ks = kFp8 ? __ldg(p.k_scale) : 1.0f;
  const float vs = kFp8 ? __ldg(p.v_scale) : 1.0f;
  const float qscale = p.qk_scale_log2 * ks;
  const QT* qp = reinterpret_cast<const QT*>(p.q);
  for (int i = tid; i < kMaxHeadsPerCta * D; i += kThreads) {
    const int h = i / D, d = i - h * D;
    q_s[i] = h < nh ? to_f32(qp[(int64_t)seq * p.q_sb + (int64_t)(h0 + h) * p.q_sh + d]) * qscale
                    : 0.0f;
  }
  if (tid < kMaxHeadsPerCta) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.0f;
  }

  const int64_t row_stride = (int64_t)p.num_kv_heads * row_bytes;  // bytes between tokens
  const int64_t head_off = (int64_t)kvh * row_bytes;
  auto load_tile = [&](int64_t t0, int stage) {
    uint8_t* kd = kbuf + stage * kGenTile * row_pitch;
    uint8_t* vd = vbuf + stage * kGenTile * row_pitch;
    for (int idx = tid; idx < kGenTile * chunks; idx += kThreads) {
      const int r = idx / chunks, c = idx - r * chunks;
      const int t = (int)t0 + r;
      int64_t page = -1;
      int blk = 0, boff = 0;
      if (t < rng.end) {
        split_token(p, t, blk, boff);
        page = page_of_block(p, seq, blk, count_invalid && c == 0);
      }
      const bool ok = page >= 0;
      const int64_t off =
          ok ? (page * p.block_size + boff) * row_stride + head_off + c * 16 : 0;
      cp_async_16(smem_u32(kd + r * row_pitch + c * 16), p.k_cache + off, ok ? 16 : 0);
      cp_async_16(smem_u32(vd + r * row_pitch + c * 16), p.v_cache + off, ok ? 16 : 0);
      if (c == 0) valid[stage * kGenTile + r] = ok ? 1 : 0;
    }
  };

  constexpr int kMaxDpt = 2;  // head_dim <= 256 = 2 columns per thread
  float acc[kMaxHeadsPerCta][kMaxDpt];
#pragma unroll
  for (int h = 0; h < kMaxHeadsPerCta; ++h)
#pragma unroll
    for (int j = 0; j < kMaxDpt; ++j) acc[h][j] = 0.0f;

  const int64_t span = rng.end > rng.begin ? rng.end - rng.begin : 0;
  const int ntiles = (int)((span + kGenTile - 1) / kGenTile);
  if (ntiles > 0) load_tile(rng.begin, 0);
  cp_async_commit();
  for (int it = 0; it < ntiles; ++it) {
    const int stage = it & 1;
    if (it + 1 < ntiles) load_tile(rng.begin + (int64_t)(it + 1) * kGenTile, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint8_t* kt = kbuf + stage * kGenTile * row_pitch;
    const uint8_t* vt = vbuf + stage * kGenTile * row_pitch;
    const uint8_t* vld = valid + stage * kGenTile;

    // scores: warp -> head, lane -> token
    for (int h = warp; h < nh; h += kThreads / 32) {
      const uint8_t* krow = kt + lane * row_pitch;
      const float* qh = q_s + h * D;
      float s = 0.0f;
      for (int c = 0; c < chunks; ++c) {
        const uint4 raw = *reinterpret_cast<const uint4*>(krow + c * 16);
        const CT* e = reinterpret_cast<const CT*>(&raw);
#pragma unroll
        for (int j = 0; j < kPer; ++j) s = fmaf(qh[c * kPer + j], to_f32(e[j]), s);
      }
      s_s[h * kGenTile + lane] = vld[lane] ? s : -INFINITY;
    }
    __syncthreads();
    // online softmax update per head (exp2 domain: q was pre-scaled by log2(e))
    for (int h = warp; h < nh; h += kThreads / 32) {
      const float s = s_s[h * kGenTile + lane];
      const float mx = warp_max(s);
      const float m_old = m_s[h];
      const float m_new = fmaxf(m_old, mx);
      const float base = m_new == -INFINITY ? 0.0f : m_new;
      const float pv = exp2f(s - base);
      const float sum = warp_sum(pv);
      s_s[h * kGenTile + lane] = pv;
      __syncwarp();
      if (lane == 0) {
        const float alpha = exp2f(m_old - base);
        a_s[h] = alpha;
        l_s[h] = l_s[h] * alpha + sum;
        m_s[h] = m_new;
      }
    }
    __syncthreads();
    // PV: thread -> output columns d = tid, tid + 128
#pragma unroll
    for (int j = 0; j < kMaxDpt; ++j) {
      const int d = tid + j * kThreads;
      if (d < D) {
#pragma unroll
        for (int h = 0; h < kMaxHeadsPerCta; ++h)
          if (h < nh) acc[h][j] *= a_s[h];
        for (int r = 0; r < kGenTile; ++r) {
          const float v = to_f32(reinterpret_cast<const CT*>(vt + r * row_pitch)[d]);
#pragma unroll
          for (int h = 0; h < kMaxHeadsPerCta; ++h)
            if (h < nh) acc[h][j] = fmaf(s_s[h * kGenTile + r], v, acc[h][j]);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  __syncthreads();

  // write the final output (single split) or this split's partial state
  const bool direct = rng.active == 1;
#pragma unroll
  for (int j = 0; j < kMaxDpt; ++j) {
    const int d = tid + j * kThreads;
    if (d >= D) continue;
#pragma unroll
    for (int h = 0; h < kMaxHeadsPerCta; ++h) {
      if (h >= nh) continue;
      const int head = h0 + h;
      if (direct) {
        QT* o = reinterpret_cast<QT*>(p.out);
        o[(int64_t)seq * p.o_sb + (int64_t)head * p.o_sh + d] =
            from_f32<QT>(acc[h][j] * vs / l_s[h]);
      } else {
        const int64_t base = ((int64_t)seq * p.num_heads + head) * p.num_splits + split;
        p.part_acc[base * D + d] = acc[h][j];
        if (d == 0) {
          p.part_ml[base * 2 + 0] = m_s[h];
          p.part_ml[base * 2 + 1] = l_s[h];
        }
      }
    }
  }
}

size_t generic_smem_bytes(int head_dim, int elem_bytes) {
  const int row_pitch = head_dim * elem_bytes + 16;
  return (size_t)4 * kGenTile * row_pitch + (size_t)kMaxHeadsPerCta * head_dim * 4 +
         (size_t)kMaxHeadsPerCta * kGenTile * 4 + 3 * kMaxHeadsPerCta * 4 + 2 * kGenTile;
}

// ============================================================ tensor-core kernel
// head_dim = 128; query bf16 with bf16 pages, f16 with f16 pages, or bf16/f16 with
// e4m3 pages (f16 MMAs). TWO_ROWS = the CTA has more than 8 query heads (MMA rows
// 8..15 in use).
template <typename CT> struct TcTraits;
template <> struct TcTraits<bf16> {
  using MT = bf16;
  static constexpr bool kFp8 = false;
  static constexpr int kStages = 3;
};
template <> struct TcTraits<f16> {
  using MT = f16;
  static constexpr bool kFp8 = false;
  static constexpr int kStages = 3;
};
template <> struct TcTraits<fp8> {
  using MT = f16;
  static constexpr bool kFp8 = true;
  static constexpr int kStages = 4;
};

constexpr int kTcD = 128;

template <typename CT>
constexpr size_t tc_smem_bytes() {
  return (size_t)TcTraits<CT>::kStages * (2 * kTcTile * kTcD * sizeof(CT) + kTcTile);
}

template <typename QT, typename CT, bool TWO_ROWS>
__global__ void __launch_bounds__(kThreads, 2)
paged_decode_tc_kernel(const DecodeParams p) {
  using Tr = TcTraits<CT>;
  using MT = typename Tr::MT;
  constexpr bool kFp8 = Tr::kFp8;
  constexpr int STAGES = Tr::kStages;
  constexpr int D = kTcD;
  constexpr int EB = sizeof(CT);
  constexpr int ROWB = D * EB;            // 256 (16-bit) or 128 (e4m3) bytes per token row
  constexpr int CPR = ROWB / 16;          // 16-byte chunks per row
  constexpr int TILE_BYTES = kTcTile * ROWB;
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  constexpr int ROWS_PER_PASS = kThreads / CPR;
  constexpr int PASSES = kTcTile / ROWS_PER_PASS;

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* valid = smem + STAGES * STAGE_BYTES;  // [STAGES][kTcTile]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.head_groups;
  const int hgrp = blockIdx.y - kvh * p.head_groups;
  const int seq = blockIdx.z;
  const int h0 = kvh * p.group + hgrp * p.heads_per_cta;
  const int nh = min(p.heads_per_cta, p.group - hgrp * p.heads_per_cta);
  const bool count_invalid = (kvh == 0 && hgrp == 0);

  const SplitRange rng = split_range(p, seq, split);
  if (split > 0 && rng.begin >= rng.end) return;
  const int64_t span = rng.end > rng.begin ? rng.end - rng.begin : 0;
  const int ntiles = (int)((span + kTcTile - 1) / kTcTile);

  // ---- producer: all threads issue 16-byte cp.async for their rows/chunks
  const int64_t row_stride = (int64_t)p.num_kv_heads * ROWB;
  const int64_t head_off = (int64_t)kvh * ROWB;
  const int ld_c = tid % CPR;
  const int ld_r0 = tid / CPR;
  // A tile never straddles a page when block_size is a power of two >= the tile.
  const bool one_page_per_tile = p.bs_shift >= 6;
  const int end = (int)rng.end;
  auto load_tile = [&](int it) {
    const int stage = it % STAGES;
    const int t0 = (int)rng.begin + it * kTcTile;
    uint8_t* kd = smem + stage * STAGE_BYTES;
    uint8_t* vd = kd + TILE_BYTES;
    int64_t tile_page = -1;
    int tile_off = 0;
    if (one_page_per_tile) {
      tile_page = page_of_block(p, seq, t0 >> p.bs_shift, count_invalid && tid == 0);
      tile_off = t0 & ((1 << p.bs_shift) - 1);
    }
#pragma unroll
    for (int i = 0; i < PASSES; ++i) {
      const int r = ld_r0 + i * ROWS_PER_PASS;
      const int t = t0 + r;
      int64_t page = -1;
      int boff = 0;
      if (t < end) {
        if (one_page_per_tile) {
          page = tile_page;
          boff = tile_off + r;
        } else {
          int blk;
          split_token(p, t, blk, boff);
          page = page_of_block(p, seq, blk, count_invalid && ld_c == 0);
        }
      }
      const bool ok = page >= 0;
      const int64_t off =
          ok ? (page * p.block_size + boff) * row_stride + head_off + ld_c * 16 : 0;
      const int soff = r * ROWB + ((ld_c ^ (r & 7)) << 4);
      cp_async_16(smem_u32(kd + soff), p.k_cache + off, ok ? 16 : 0);
      cp_async_16(smem_u32(vd + soff), p.v_cache + off, ok ? 16 : 0);
      if (ld_c == 0) valid[stage * kTcTile + r] = ok ? 1 : 0;
    }
  };

  // prologue: put STAGES-1 tiles in flight before building the query fragments
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < ntiles) load_tile(s);
    cp_async_commit();
  }

  // ---- query fragments (A operand, rows = query heads of this CTA)
  const QT* qp = reinterpret_cast<const QT*>(p.q);
  auto qval = [&](int row, int d) -> float {
    return row < nh ? to_f32(qp[(int64_t)seq * p.q_sb + (int64_t)(h0 + row) * p.q_sh + d]) : 0.0f;
  };
  // column of element j (0..3) of row-fragment half `hi` for k-step ks
  // 16-bit pages: a0 = cols 2tig,2tig+1; a2 = cols 8+2tig, 8+2tig+1 (PTX m16n8k16 layout)
  // e4m3 pages: k index kappa -> d permuted so one ldmatrix word (4 bytes = d 4tig..4tig+3)
  //             feeds b0 (kappa 2tig,2tig+1) and b1 (kappa 2tig+8, 2tig+9).
  auto qcol = [&](int ks, int half, int e) -> int {
    if (kFp8) return 16 * ks + 4 * tig + 2 * half + e;
    return 16 * ks + 8 * half + 2 * tig + e;
  };
  float qpow2 = 1.0f;  // FP8 path: bf16 query rescaled by a power of two into f16 range
  if (kFp8 && std::is_same<QT, bf16>::value) {
    float mx = 0.0f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
      for (int half = 0; half < 2; ++half)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          mx = fmaxf(mx, fabsf(qval(g, qcol(ks, half, e))));
          if (TWO_ROWS) mx = fmaxf(mx, fabsf(qval(g + 8, qcol(ks, half, e))));
        }
    mx = warp_max(mx);
    if (mx > 0.0f && isfinite(mx)) {
      int ex;
      frexpf(mx, &ex);            // mx = f * 2^ex, f in [0.5, 1)
      qpow2 = ldexpf(1.0f, 15 - ex);  // max |q| * qpow2 < 2^15 < f16 max
    }
  }
  uint32_t qa[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    qa[ks][0] = pack2<MT>(qval(g, qcol(ks, 0, 0)) * qpow2, qval(g, qcol(ks, 0, 1)) * qpow2);
    qa[ks][2] = pack2<MT>(qval(g, qcol(ks, 1, 0)) * qpow2, qval(g, qcol(ks, 1, 1)) * qpow2);
    if (TWO_ROWS) {
      qa[ks][1] =
          pack2<MT>(qval(g + 8, qcol(ks, 0, 0)) * qpow2, qval(g + 8, qcol(ks, 0, 1)) * qpow2);
      qa[ks][3] =
          pack2<MT>(qval(g + 8, qcol(ks, 1, 0)) * qpow2, qval(g + 8, qcol(ks, 1, 1)) * qpow2);
    } else {
      qa[ks][1] = 0u;
      qa[ks][3] = 0u;
    }
  }
  const float ks_scale = kFp8 ? __ldg(p.k_scale) : 1.0f;
  const float vs_scale = kFp8 ? __ldg(p.v_scale) : 1.0f;
  const float sc = p.qk_scale_log2 * ks_scale / qpow2;

  // ---- per-warp softmax state (rows g and g+8) and output accumulators
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;

  const int lrow = lane & 7;   // ldmatrix: row within the 8x8 matrix this lane addresses
  const int lmat = lane >> 3;  // ldmatrix: which of the 4 matrices
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (it + STAGES - 1 < ntiles) load_tile(it + STAGES - 1);
    cp_async_commit();

    const int stage = it % STAGES;
    const uint8_t* kt = smem + stage * STAGE_BYTES;
    const uint8_t* vt = kt + TILE_BYTES;
    const uint8_t* vld = valid + stage * kTcTile;
    const uint32_t kbase = smem_u32(kt);
    const uint32_t vbase = smem_u32(vt);

    // ---- S = Q K^T for this warp's 16 tokens (two n8 tiles)
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
      const int r = warp * 16 + nt * 8 + lrow;
      if (!kFp8) {
#pragma unroll
        for (int kp = 0; kp < D / 32; ++kp) {
          const int lc = 4 * kp + lmat;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kbase + r * ROWB + ((lc ^ lrow) << 4), b0, b1, b2, b3);
          Mma<MT>::run(s[nt], qa[2 * kp], b0, b1);
          Mma<MT>::run(s[nt], qa[2 * kp + 1], b2, b3);
        }
      } else {
#pragma unroll
        for (int kq = 0; kq < D / 64; ++kq) {
          const int lc = 4 * kq + lmat;
          uint32_t x[4];
          ldmatrix_x4(kbase + r * ROWB + ((lc ^ lrow) << 4), x[0], x[1], x[2], x[3]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t b0 = e4m3x2_to_f16x2((uint16_t)(x[j] & 0xffffu));
            const uint32_t b1 = e4m3x2_to_f16x2((uint16_t)(x[j] >> 16));
            Mma<MT>::run(s[nt], qa[4 * kq + j], b0, b1);
          }
        }
      }
    }

    // ---- online softmax (exp2 domain)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int tok = warp * 16 + nt * 8 + 2 * tig;
      const bool v0 = vld[tok] != 0, v1 = vld[tok + 1] != 0;
      s[nt][0] = v0 ? s[nt][0] * sc : -INFINITY;
      s[nt][1] = v1 ? s[nt][1] * sc : -INFINITY;
      s[nt][2] = v0 ? s[nt][2] * sc : -INFINITY;
      s[nt][3] = v1 ? s[nt][3] * sc : -INFINITY;
    }
    float p[2][4];
    {
      float mx = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m0, mx);
      const float base = m_new == -INFINITY ? 0.0f : m_new;
      const float alpha = exp2f(m0 - base);
      m0 = m_new;
      p[0][0] = exp2f(s[0][0] - base);
      p[0][1] = exp2f(s[0][1] - base);
      p[1][0] = exp2f(s[1][0] - base);
      p[1][1] = exp2f(s[1][1] - base);
      l0 = l0 * alpha + ((p[0][0] + p[0][1]) + (p[1][0] + p[1][1]));
      if (alpha != 1.0f) {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[n][0] *= alpha;
          o[n][1] *= alpha;
        }
      }
    }
    if (TWO_ROWS) {
      float mx = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m1, mx);
      const float base = m_new == -INFINITY ? 0.0f : m_new;
      const float alpha = exp2f(m1 - base);
      m1 = m_new;
      p[0][2] = exp2f(s[0][2] - base);
      p[0][3] = exp2f(s[0][3] - base);
      p[1][2] = exp2f(s[1][2] - base);
      p[1][3] = exp2f(s[1][3] - base);
      l1 = l1 * alpha + ((p[0][2] + p[0][3]) + (p[1][2] + p[1][3]));
      if (alpha != 1.0f) {
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[n][2] *= alpha;
          o[n][3] *= alpha;
        }
      }
    } else {
      p[0][2] = p[0][3] = p[1][2] = p[1][3] = 0.0f;
    }

    // ---- O += P V (P as the A operand straight from the S accumulator layout)
    uint32_t pa[4];
    pa[0] = pack2<MT>(p[0][0], p[0][1]);
    pa[1] = pack2<MT>(p[0][2], p[0][3]);
    pa[2] = pack2<MT>(p[1][0], p[1][1]);
    pa[3] = pack2<MT>(p[1][2], p[1][3]);
    const int vr = warp * 16 + ((lmat & 1) << 3) + lrow;  // token row this lane addresses
    if (!kFp8) {
#pragma unroll
      for (int cp = 0; cp < D / 16; ++cp) {
        const int lc = 2 * cp + (lmat >> 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vbase + vr * ROWB + ((lc ^ lrow) << 4), b0, b1, b2, b3);
        Mma<MT>::run(o[2 * cp], pa, b0, b1);
        Mma<MT>::run(o[2 * cp + 1], pa, b2, b3);
      }
    } else {
      // ldmatrix.trans over e4m3 rows gives, per register, tokens (2tig, 2tig+1) x
      // d (2g, 2g+1) of a 16-column chunk; a byte permute splits even and odd d.
#pragma unroll
      for (int cq = 0; cq < D / 32; ++cq) {
        const int lc = 2 * cq + (lmat >> 1);
        uint32_t x[4];
        ldmatrix_x4_trans(vbase + vr * ROWB + ((lc ^ lrow) << 4), x[0], x[1], x[2], x[3]);
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {  // chunk 2cq + hc: x[2hc] tokens 0-7, x[2hc+1] tokens 8-15
          const uint32_t lo = __byte_perm(x[2 * hc], 0u, 0x3120);
          const uint32_t hi = __byte_perm(x[2 * hc + 1], 0u, 0x3120);
          Mma<MT>::run(o[4 * cq + 2 * hc + 0], pa, e4m3x2_to_f16x2((uint16_t)(lo & 0xffffu)),
                       e4m3x2_to_f16x2((uint16_t)(hi & 0xffffu)));
          Mma<MT>::run(o[4 * cq + 2 * hc + 1], pa, e4m3x2_to_f16x2((uint16_t)(lo >> 16)),
                       e4m3x2_to_f16x2((uint16_t)(hi >> 16)));
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- merge the 4 warps' states through shared memory (reusing the ring)
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  if (TWO_ROWS) {
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  }
  constexpr int RP = D + 4;  // padded row pitch (floats)
  float* red_acc = reinterpret_cast<float*>(smem);               // [4][16][RP]
  float* red_m = red_acc + 4 * kMaxHeadsPerCta * RP;             // [4][16]
  float* red_l = red_m + 4 * kMaxHeadsPerCta;                    // [4][16]
  static_assert((4 * kMaxHeadsPerCta * RP + 8 * kMaxHeadsPerCta) * 4 <= STAGES * STAGE_BYTES,
                "merge buffer fits in the ring");
  auto out_col = [&](int n, int e) -> int {  // column of accumulator o[n][e] / o[n][e+2]
    if (kFp8) {
      const int chunk = n >> 1, odd = n & 1;
      return 16 * chunk + 4 * tig + 2 * e + odd;
    }
    return 8 * n + 2 * tig + e;
  };
  {
    float* ra = red_acc + (warp * kMaxHeadsPerCta + g) * RP;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      ra[out_col(n, 0)] = o[n][0];
      ra[out_col(n, 1)] = o[n][1];
    }
    if (tig == 0) {
      red_m[warp * kMaxHeadsPerCta + g] = m0;
      red_l[warp * kMaxHeadsPerCta + g] = l0;
    }
    if (TWO_ROWS) {
      float* rb = red_acc + (warp * kMaxHeadsPerCta + g + 8) * RP;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        rb[out_col(n, 0)] = o[n][2];
        rb[out_col(n, 1)] = o[n][3];
      }
      if (tig == 0) {
        red_m[warp * kMaxHeadsPerCta + g + 8] = m1;
        red_l[warp * kMaxHeadsPerCta + g + 8] = l1;
      }
    }
  }
  __syncthreads();

  const bool direct = rng.active == 1;
  for (int idx = tid; idx < nh * D; idx += kThreads) {
    const int h = idx / D, d = idx - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red_m[w * kMaxHeadsPerCta + h]);
    const float base = M == -INFINITY ? 0.0f : M;
    float O = 0.0f, L = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float wgt = exp2f(red_m[w * kMaxHeadsPerCta + h] - base);
      O = fmaf(wgt, red_acc[(w * kMaxHeadsPerCta + h) * RP + d], O);
      L = fmaf(wgt, red_l[w * kMaxHeadsPerCta + h], L);
    }
    const int head = h0 + h;
    if (direct) {
      QT* op = reinterpret_cast<QT*>(p.out);
      op[(int64_t)seq * p.o_sb + (int64_t)head * p.o_sh + d] = from_f32<QT>(O * vs_scale / L);
    } else {
      const int64_t b = ((int64_t)seq * p.num_heads + head) * p.num_splits + split;
      p.part_acc[b * D + d] = O;
      if (d == 0) {
        p.part_ml[b * 2 + 0] = M;
        p.part_ml[b * 2 + 1] = L;
      }
    }
  }
}

// ============================================================ split merge
// One CTA per (head, sequence): combines the active splits' (m, l, acc) and writes
// out = (sum_s 2^(m_s - M) acc_s) * v_scale / (sum_s 2^(m_s - M) l_s).
template <typename QT>
__global__ void __launch_bounds__(kThreads) split_merge_kernel(const DecodeParams p) {
  const int head = blockIdx.x, seq = blockIdx.y;
  const SplitRange rng = split_range(p, seq, 0);
  if (rng.active <= 1) return;  // written directly by the split kernel
  const int64_t base = ((int64_t)seq * p.num_heads + head) * p.num_splits;
  __shared__ float wts[512];
  __shared__ float sh_l;
  float M = -INFINITY;
  for (int s = 0; s < rng.active; ++s) M = fmaxf(M, p.part_ml[(base + s) * 2]);
  const float mb = M == -INFINITY ? 0.0f : M;
  for (int s = threadIdx.x; s < rng.active; s += blockDim.x)
    wts[s] = exp2f(p.part_ml[(base + s) * 2] - mb);
  __syncthreads();
  if (threadIdx.x == 0) {
    float L = 0.0f;
    for (int s = 0; s < rng.active; ++s) L = fmaf(wts[s], p.part_ml[(base + s) * 2 + 1], L);
    sh_l = L;
  }
  __syncthreads();
  const float vs = p.v_scale != nullptr ? __ldg(p.v_scale) : 1.0f;
  const float L = sh_l;
  QT* op = reinterpret_cast<QT*>(p.out);
  for (int d = threadIdx.x; d < p.head_dim; d += blockDim.x) {
    float O = 0.0f;
    for (int s = 0; s < rng.active; ++s) O = fmaf(wts[s], p.part_acc[(base + s) * p.head_dim + d], O);
    op[(int64_t)seq * p.o_sb + (int64_t)head * p.o_sh + d] = from_f32<QT>(O * vs / L);
  }
}

constexpr int kMaxSplits = 512;  // split_merge_kernel's weight buffer

// ============================================================ host side
struct SplitPlan {
  int num_splits;
  int chunk;
};

inline int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// Shapes only: the number of CTAs per (seq, kv head) is sized so the grid covers
// several waves of the 148 SMs at two resident CTAs each, with chunks of at most 1024
// tokens (balanced work for ragged batches) and at least 128 tokens.
SplitPlan plan_splits(int num_seqs, int num_kv_heads, int head_groups, int block_size,
                      int max_blocks, int forced) {
  SplitPlan sp;
  const int64_t cap = (int64_t)max_blocks * block_size;
  if (cap <= 0) {
    sp.num_splits = 1;
    sp.chunk = kChunkAlign;
    return sp;
  }
  int64_t chunk;
  if (forced > 0) {
    chunk = round_up((cap + forced - 1) / forced, kChunkAlign);
  } else {
    const int64_t units = (int64_t)num_seqs * num_kv_heads * head_groups;
    const int64_t target = (int64_t)kNumSMs * 2 * 8;
    chunk = 1024;
    while (chunk > 128 && units * ((cap + chunk - 1) / chunk) < target) chunk /= 2;
  }
  if (chunk >= cap) chunk = round_up(cap, kChunkAlign);
  int64_t n = (cap + chunk - 1) / chunk;
  if (n > kMaxSplits) {
    chunk = round_up((cap + kMaxSplits - 1) / kMaxSplits, kChunkAlign);
    n = (cap + chunk - 1) / chunk;
  }
  sp.num_splits = (int)n;
  sp.chunk = (int)chunk;
  return sp;
}

int head_groups_for(int group) { return (group + kMaxHeadsPerCta - 1) / kMaxHeadsPerCta; }

size_t workspace_bytes_for(int num_seqs, int num_heads, int head_dim, int num_splits) {
  if (num_splits <= 1) return 0;
  const size_t n = (size_t)num_seqs * num_heads * num_splits;
  const size_t acc = round_up((int64_t)(n * head_dim * sizeof(float)), 256);
  return acc + n * 2 * sizeof(float);
}

// One cudaFuncSetAttribute per kernel instantiation and device.
template <auto Kernel>
int ensure_smem(size_t bytes, int device) {
  static unsigned long long configured = 0;  // bit per device id < 64
  if (bytes <= 48 * 1024) return MKV_OK;
  const unsigned long long bit = device < 64 ? (1ull << device) : 0ull;
  if (bit && (__atomic_load_n(&configured, __ATOMIC_RELAXED) & bit)) return MKV_OK;
  cudaError_t e =
      cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(max dynamic smem)");
  if (bit) __atomic_fetch_or(&configured, bit, __ATOMIC_RELAXED);
  return MKV_OK;
}

template <typename QT, typename CT>
int launch_generic(const DecodeParams& p, dim3 grid, cudaStream_t stream, int device) {
  const size_t smem = generic_smem_bytes(p.head_dim, sizeof(CT));
  // opt in once to the largest size this instantiation can use (head_dim 256)
  int st = ensure_smem<paged_decode_generic_kernel<QT, CT>>(generic_smem_bytes(256, sizeof(CT)),
                                                            device);
  if (st != MKV_OK) return st;
  paged_decode_generic_kernel<QT, CT><<<grid, kThreads, smem, stream>>>(p);
  return cuda_status(cudaGetLastError(), "paged_decode_generic launch");
}

template <typename QT, typename CT>
int launch_tc(const DecodeParams& p, dim3 grid, cudaStream_t stream, int device) {
  constexpr size_t smem = tc_smem_bytes<CT>();
  if (p.heads_per_cta > 8) {
    int st = ensure_smem<paged_decode_tc_kernel<QT, CT, true>>(smem, device);
    if (st != MKV_OK) return st;
    paged_decode_tc_kernel<QT, CT, true><<<grid, kThreads, smem, stream>>>(p);
  } else {
    int st = ensure_smem<paged_decode_tc_kernel<QT, CT, false>>(smem, device);
    if (st != MKV_OK) return st;
    paged_decode_tc_kernel<QT, CT, false><<<grid, kThreads, smem, stream>>>(p);
  }
  return cuda_status(cudaGetLastError(), "paged_decode_tc launch");
}

template <typename QT>
int launch_merge(const DecodeParams& p, cudaStream_t stream) {
  dim3 grid(p.num_heads, p.num_seqs);
  split_merge_kernel<QT><<<grid, kThreads, 0, stream>>>(p);
  return cuda_status(cudaGetLastError(), "split_merge launch");
}

int decode_impl(const char* fn, const void* query, int64_t q_sb, int64_t q_sh, int q_dtype,
                const void* k_cache, const void* v_cache, int cache_dtype, const float* k_scale,
                const float* v_scale, int64_t num_blocks, int block_size, const void* bt,
                int bt_type, int64_t bt_sb, int max_blocks, const void* ctx, int ctx_type,
                int num_seqs, int num_heads, int num_kv_heads, int head_dim, float scale,
                void* out, int64_t o_sb, int64_t o_sh, void* workspace, size_t ws_bytes,
                int num_splits, int32_t* invalid, void* stream) {
  clear_error();
  if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 ||
      max_blocks < 0 || num_blocks < 0 || num_splits < 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "%s: bad sizes (num_seqs=%d num_heads=%d num_kv_heads=%d head_dim=%d "
                     "block_size=%d max_num_blocks=%d num_blocks=%lld num_splits=%d)",
                     fn, num_seqs, num_heads, num_kv_heads, head_dim, block_size, max_blocks,
                     (long long)num_blocks, num_splits);
  if (num_heads % num_kv_heads != 0)
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "%s: num_heads (%d) must be a multiple of num_kv_heads (%d)", fn, num_heads,
                     num_kv_heads);
  if (bt_type != MKV_INDEX_I32 && bt_type != MKV_INDEX_I64)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: bad block_table_index_type", fn);
  if (ctx_type != MKV_INDEX_I32 && ctx_type != MKV_INDEX_I64)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: bad context_lens_index_type", fn);
  if (num_seqs == 0) return MKV_OK;
  if (!query || !k_cache || !v_cache || !ctx || !out || (max_blocks > 0 && !bt))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (num_seqs > 65535)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: num_seqs > 65535", fn);
  if ((int64_t)max_blocks * block_size >= ((int64_t)1 << 31))
    return set_error(MKV_ERR_UNSUPPORTED, "%s: max_num_blocks * block_size must be < 2^31", fn);
  if (head_dim % 16 != 0 || head_dim > 256)
    return set_error(MKV_ERR_UNSUPPORTED,
                     "%s: head_dim must be a multiple of 16 and at most 256 (got %d)", fn,
                     head_dim);
  const bool fp8_cache = cache_dtype == MKV_DTYPE_FP8_E4M3;
  if (fp8_cache && (!k_scale || !v_scale))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: FP8 cache needs k_scale and v_scale", fn);
  if (!fp8_cache && cache_dtype != q_dtype)
    return set_error(MKV_ERR_UNSUPPORTED,
                     "%s: cache dtype (%d) must equal the query dtype (%d) for float caches", fn,
                     cache_dtype, q_dtype);
  if (q_dtype != MKV_DTYPE_F32 && q_dtype != MKV_DTYPE_F16 && q_dtype != MKV_DTYPE_BF16)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: query dtype must be f32, f16 or bf16", fn);
  if (((uintptr_t)k_cache & 15u) || ((uintptr_t)v_cache & 15u))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: caches must be 16-byte aligned", fn);

  const int group = num_heads / num_kv_heads;
  const int hpc = group < kMaxHeadsPerCta ? group : kMaxHeadsPerCta;
  const int hgs = head_groups_for(group);
  if ((int64_t)num_kv_heads * hgs > 65535)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: too many kv heads", fn);
  const SplitPlan sp = plan_splits(num_seqs, num_kv_heads, hgs, block_size, max_blocks, num_splits);
  const size_t need = workspace_bytes_for(num_seqs, num_heads, head_dim, sp.num_splits);
  if (need > 0 && (workspace == nullptr || ws_bytes < need))
    return set_error(MKV_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn, need,
                     workspace ? ws_bytes : (size_t)0);
  if (need > 0 && ((uintptr_t)workspace & 15u))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: workspace must be 16-byte aligned", fn);

  DecodeParams p;
  p.q = query;
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  p.k_cache = (const uint8_t*)k_cache;
  p.v_cache = (const uint8_t*)v_cache;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctz((unsigned)block_size) : -1;
  p.bt = bt;
  p.bt_sb = bt_sb;
  p.max_blocks = max_blocks;
  p.bt_i64 = bt_type == MKV_INDEX_I64;
  p.ctx = ctx;
  p.ctx_i64 = ctx_type == MKV_INDEX_I64;
  p.num_seqs = num_seqs;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.group = group;
  p.heads_per_cta = hpc;
  p.head_groups = hgs;
  p.qk_scale_log2 = scale * kLog2e;
  p.k_scale = fp8_cache ? k_scale : nullptr;
  p.v_scale = fp8_cache ? v_scale : nullptr;
  p.out = out;
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.num_splits = sp.num_splits;
  p.chunk = sp.chunk;
  p.part_acc = need > 0 ? (float*)workspace : nullptr;
  p.part_ml = need > 0 ? (float*)((uint8_t*)workspace +
                                  round_up((int64_t)((size_t)num_seqs * num_heads * sp.num_splits *
                                                     head_dim * sizeof(float)),
                                           256))
                       : nullptr;
  p.invalid = invalid;

  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  cudaStream_t s = (cudaStream_t)stream;
  dim3 grid(sp.num_splits, num_kv_heads * hgs, num_seqs);

  const bool tc_ok = head_dim == kTcD && q_dtype != MKV_DTYPE_F32;
  int st;
  if (tc_ok && !fp8_cache && q_dtype == MKV_DTYPE_BF16)
    st = launch_tc<bf16, bf16>(p, grid, s, device);
  else if (tc_ok && !fp8_cache && q_dtype == MKV_DTYPE_F16)
    st = launch_tc<f16, f16>(p, grid, s, device);
  else if (tc_ok && fp8_cache && q_dtype == MKV_DTYPE_BF16)
    st = launch_tc<bf16, fp8>(p, grid, s, device);
  else if (tc_ok && fp8_cache && q_dtype == MKV_DTYPE_F16)
    st = launch_tc<f16, fp8>(p, grid, s, device);
  else if (fp8_cache) {
    switch (q_dtype) {
      case MKV_DTYPE_F32: st = launch_generic<float, fp8>(p, grid, s, device); break;
      case MKV_DTYPE_F16: st = launch_generic<f16, fp8>(p, grid, s, device); break;
      default: st = launch_generic<bf16, fp8>(p, grid, s, device); break;
    }
  } else {
    switch (q_dtype) {
      case MKV_DTYPE_F32: st = launch_generic<float, float>(p, grid, s, device); break;
      case MKV_DTYPE_F16: st = launch_generic<f16, f16>(p, grid, s, device); break;
      default: st = launch_generic<bf16, bf16>(p, grid, s, device); break;
    }
  }
  if (st != MKV_OK || sp.num_splits <= 1) return st;
  switch (q_dtype) {
    case MKV_DTYPE_F32: return launch_merge<float>(p, s);
    case MKV_DTYPE_F16: return launch_merge<f16>(p, s);
    default: return launch_merge<bf16>(p, s);
  }
}

}  // namespace
}  // namespace mkv

using namespace mkv;

extern "C" int32_t mkv_paged_decode_num_splits(int32_t num_seqs, int32_t num_heads,
                                               int32_t num_kv_heads, int32_t head_dim,
                                               int32_t block_size, int32_t max_num_blocks) {
  (void)head_dim;
  if (num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads != 0) return 1;
  const int hgs = head_groups_for(num_heads / num_kv_heads);
  return plan_splits(num_seqs, num_kv_heads, hgs, block_size, max_num_blocks, 0).num_splits;
}

extern "C" size_t mkv_paged_decode_workspace_bytes(int32_t num_seqs, int32_t num_heads,
                                                   int32_t num_kv_heads, int32_t head_dim,
                                                   int32_t block_size, int32_t max_num_blocks,
                                                   int32_t num_splits) {
  if (num_seqs <= 0 || num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads != 0 ||
      head_dim <= 0 || num_splits < 0)
    return 0;
  const int hgs = head_groups_for(num_heads / num_kv_heads);
  const SplitPlan sp =
      plan_splits(num_seqs, num_kv_heads, hgs, block_size, max_num_blocks, num_splits);
  return workspace_bytes_for(num_seqs, num_heads, head_dim, sp.num_splits);
}

extern "C" int mkv_paged_decode(const void* query, int64_t q_stride_seq, int64_t q_stride_head,
                                int32_t q_dtype, const void* k_cache, const void* v_cache,
                                int32_t cache_dtype, int64_t num_blocks, int32_t block_size,
                                const void* block_tables, int32_t block_table_index_type,
                                int64_t block_table_stride_seq, int32_t max_num_blocks,
                                const void* context_lens, int32_t context_lens_index_type,
                                int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                int32_t head_dim, float scale, void* out, int64_t out_stride_seq,
                                int64_t out_stride_head, void* workspace, size_t workspace_bytes,
                                int32_t num_splits, int32_t* invalid_count, void* stream) {
  if (cache_dtype == MKV_DTYPE_FP8_E4M3)
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "mkv_paged_decode: FP8 caches go through mkv_paged_decode_fp8");
  return decode_impl("mkv_paged_decode", query, q_stride_seq, q_stride_head, q_dtype, k_cache,
                     v_cache, cache_dtype, nullptr, nullptr, num_blocks, block_size, block_tables,
                     block_table_index_type, block_table_stride_seq, max_num_blocks, context_lens,
                     context_lens_index_type, num_seqs, num_heads, num_kv_heads, head_dim, scale,
                     out, out_stride_seq, out_stride_head, workspace, workspace_bytes, num_splits,
                     invalid_count, stream);
}

extern "C" int mkv_paged_decode_fp8(const void* query, int64_t q_stride_seq,
                                    int64_t q_stride_head, int32_t q_dtype, const void* k_cache,
                                    const void* v_cache, const float* k_scale,
                                    const float* v_scale, int64_t num_blocks, int32_t block_size,
                                    const void* block_tables, int32_t block_table_index_type,
                                    int64_t block_table_stride_seq, int32_t max_num_blocks,
                                    const void* context_lens, int32_t context_lens_index_type,
                                    int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                    int32_t head_dim, float scale, void* out,
                                    int64_t out_stride_seq, int64_t out_stride_head,
                                    void* workspace, size_t workspace_bytes, int32_t num_splits,
                                    int32_t* invalid_count, void* stream) {
  return decode_impl("mkv_paged_decode_fp8", query, q_stride_seq, q_stride_head, q_dtype, k_cache,
                     v_cache, MKV_DTYPE_FP8_E4M3, k_scale, v_scale, num_blocks, block_size,
                     block_tables, block_table_index_type, block_table_stride_seq, max_num_blocks,
                     context_lens, context_lens_index_type, num_seqs, num_heads, num_kv_heads,
                     head_dim, scale, out, out_stride_seq, out_stride_head, workspace,
                     workspace_bytes, num_splits, invalid_count, stream);
}
