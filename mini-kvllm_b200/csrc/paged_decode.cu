// Paged-attention decode: one query token per sequence against its paged K/V.
//
// Reference behaviour (heart1128/mini-kvllm, src/myvllm/layers/attention.py):
//   paged_attention_decode_kernel      attention.py:517-646  (bf16/fp16/fp32 cache)
//   paged_attention_decode_fp8_kernel  attention.py:953-1121 (PER_TOKEN_HEAD=0: per-tensor scales)
//   wrappers                           attention.py:895-950, 1213-1268
// Semantics kept: kv_head = h / (H / KVH); tokens t < context_len whose logical block
// t / block_size is < max_num_blocks; page = block_tables[b, t / block_size] with -1
// meaning "skip this token"; FP8 values dequantised as float(e4m3) * scale; output
// = softmax(scale * q.K) V in fp32, stored in the query dtype; no visible token -> NaN.
//
// B200 design (HBM-bound: ~2 * G FLOP per cache byte):
//   * a CTA works on (sequence, kv head) units and covers the whole GQA group, so each
//     page row is read from HBM once, not G times as in the reference's (seq, head) grid;
//   * pages stream through a multi-stage cp.async ring of 64-token tiles in shared
//     memory (16-byte chunks, XOR-swizzled so ldmatrix reads are conflict-free); the
//     CTA's block-table slice is staged in shared memory first;
//   * QK^T and PV run on the tensor cores (mma.sync m16n8k16, fp32 accumulate) in the
//     transposed form S^T = K Q^T and O^T = V^T P^T: the 16 tokens of a warp are the
//     M rows and the query group (padded to 8) is N, so no MMA row is wasted on
//     padding heads. P^T is re-laid out as the B operand with movmatrix.trans;
//   * FP8 pages are converted e4m3x2 -> f16x2 in registers straight out of ldmatrix
//     (head_dim permuted so one ldmatrix word feeds both halves of a fragment), so
//     dequantisation adds no memory traffic; the K scale is folded into the score
//     scale and V's into the output;
//   * online softmax in the exp2 domain; 4 warps split each tile and merge their
//     (m, l, acc) through shared memory at the end;
//   * balanced persistent schedule (num_splits = 0): the grid is the kernel's resident
//     CTAs (occupancy x SMs) and each CTA reads the context lengths once and takes an
//     equal share of all (unit, tile) work items, so ragged batches and uniform long
//     contexts both load every SM evenly, with no wave tail and no per-chunk restart.
//     A unit that crosses a CTA boundary is finished by partials: each writes
//     (m, l, acc) to the workspace and bumps the unit's counter; the last to arrive
//     merges them and writes the output, so there is no second kernel. A forced
//     num_splits > 0 instead splits every unit into fixed token chunks (flash-decoding)
//     with the same epilogue. Nothing on the host depends on device data (graph-safe).
// A CUDA-core kernel with the same tiling and epilogue covers fp32 and other head dims.
#include <mutex>
#include <type_traits>

#include "mkv_common.cuh"

namespace mkv {
namespace {

constexpr int kThreads = 128;        // 4 warps per CTA (both kernels)
constexpr int kMaxHeadsPerCta = 16;  // query heads of one KV head handled by a CTA
constexpr int kTcTile = 64;          // tokens per pipeline stage, tensor-core kernel
constexpr int kGenTile = 32;         // tokens per pipeline stage, CUDA-core kernel
constexpr int kChunkAlign = 128;     // split boundaries are multiples of every tile
constexpr int kMaxSplits = 128;     // bounds the partials a unit is merged from
constexpr int kMaxBtSmem = 128;      // block-table entries staged in shared memory
constexpr int kTcD = 128;           // head_dim of the tensor-core kernels
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
  float qk_scale_log2;   // attention scale * log2(e)
  const float* k_scale;  // FP8 per-tensor scales (nullptr for float caches)
  const float* v_scale;
  // per-(page, row, kv head) scales of 8-bit caches, (num_blocks, block_size, kv heads)
  const float* k_scales;
  const float* v_scales;
  void* out;
  int64_t o_sb, o_sh;  // elements
  float* part_acc;     // [num_seqs][num_heads][num_splits][head_dim]
  float* part_ml;      // [num_seqs][num_heads][num_splits][2] = (m in log2 units, l)
  unsigned int* arrivals;  // [num_seqs][num_kv_heads * head_groups], zero between launches
  int num_splits;
  int chunk;  // tokens per split, multiple of kChunkAlign
  // Balanced schedule (num_splits = 0): the grid is sched_ctas resident CTAs and each
  // takes an equal share of all (unit, tile) work items; every CTA gets >= min_tiles.
  int balanced;
  int sched_ctas;
  int min_tiles;
  int unit_cost;  // balanced: items charged per unit before its tiles (segment overhead)
  int q_vec16;  // query rows start on 16-byte boundaries (base and both strides)
  int32_t* invalid;
  int pdl;  // host only: launch with programmatic stream serialization
};

__device__ __forceinline__ int64_t load_ctx(const DecodeParams& p, int seq) {
  return p.ctx_i64 ? (int64_t)__ldg((const int64_t*)p.ctx + seq)
                   : (int64_t)__ldg((const int32_t*)p.ctx + seq);
}

// Validated page of logical block `blk` of sequence `seq`: -1 when the entry is -1 or
// outside [0, num_blocks); such out-of-range entries (other than -1) are counted.
__device__ __forceinline__ int page_of_block(const DecodeParams& p, int seq, int blk, bool count) {
  const int64_t idx = (int64_t)seq * p.bt_sb + blk;
  const int64_t page = p.bt_i64 ? (int64_t)__ldg((const int64_t*)p.bt + idx)
                                : (int64_t)__ldg((const int32_t*)p.bt + idx);
  if (page >= 0 && page < p.num_blocks) return (int)page;
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
  int begin, end, active;
};
__device__ __forceinline__ SplitRange split_range(const DecodeParams& p, int seq, int split) {
  const int64_t ctx = load_ctx(p, seq);
  const int64_t cap = (int64_t)p.max_blocks * p.block_size;
  int64_t eff = ctx < cap ? ctx : cap;
  if (eff < 0) eff = 0;
  SplitRange r;
  r.active = eff > 0 ? (int)((eff + p.chunk - 1) / p.chunk) : 1;
  r.begin = split * p.chunk;
  r.end = (int)((int64_t)r.begin + p.chunk < eff ? (int64_t)r.begin + p.chunk : eff);
  return r;
}


// ---------------------------------------------------------------- work schedule
// A unit is (sequence, KV head, head group): y = kv_head * head_groups + head group.
// A segment is a contiguous token range of one unit processed by one CTA. With a fixed
// split count (num_splits > 0) a CTA runs the single segment (split, y, seq) of its
// grid coordinates. With the balanced schedule the work items (token tiles) are split
// evenly over the CTAs, each taking a contiguous range and so walking one or more
// segments; a unit that crosses a CTA boundary is finished by partials.
//   * Lanes (the U = kv_heads * head_groups values of y share the grid evenly): CTA
//     c = y + U * r is rank r of lane y; lane y's items are the tiles of units (s, y) for
//     s = 0, 1, ... and its G/U ranks split them evenly. All lanes walk the same token
//     ranges at the same pace, so the KV heads of a token row (adjacent in HBM) are read
//     together, as with a fixed (split, head, seq) grid.
//   * Otherwise (U does not divide the grid closely enough) one sequence of W items over
//     all units, sequence-major, split over the G CTAs.
// Rank r's range is [W*r/G, W*(r+1)/G) in its item sequence. Partial k of a unit is
// written by rank r_first + k, i.e. CTA cta_base + cta_stride*(r_first + k), into slot
// 2*cta + (k == 0 ? first_off : 0): slot 2c holds CTA c's first segment, 2c+1 its last,
// so every slot has one writer and the workspace is bounded by 2 * grid slots.
struct TokRange {
  int begin, end;
};
struct Seg {
  int seq, y;
  int begin, end;  // token range [begin, end)
  int nparts;      // partials of the unit (1 = this segment is the whole unit)
  int part;        // this segment's index among them
  int c_first, first_off;   // rank of partial 0's writer; partial 0 in its last-segment slot
  int cta_base, cta_stride; // CTA index of rank r: cta_base + cta_stride * r
};

__device__ __forceinline__ int eff_ctx(const DecodeParams& p, int seq) {
  const int64_t ctx = load_ctx(p, seq);
  const int64_t cap = (int64_t)p.max_blocks * p.block_size;
  const int64_t eff = ctx < cap ? ctx : cap;
  return eff > 0 ? (int)eff : 0;
}
// Tiles of one unit of the sequence; an empty context still takes one (empty) tile so
// that its output (0/0 = NaN, as in the reference) is written.
template <int TILE>
__device__ __forceinline__ int unit_tiles(int eff) { return eff > 0 ? (eff + TILE - 1) / TILE : 1; }

// Schedule state, uniform across the CTA, kept in shared memory so the kernels' inner
// loops carry none of it in registers. Thread 0 advances it between two barriers.
struct SchedState {
  long long w, w_end, unit_start, W, G;  // item range of this rank; items and ranks in its sequence
  int seq, y, nt, eff, U;
  int lanes, rank;
  int has, fixed_pending;
  Seg cur;
};

// CTA of work item x: the largest c with W*c/G <= x.
__device__ __forceinline__ long long cta_of(const SchedState& st, long long x) {
  return ((x + 1) * st.G - 1) / st.W;
}

// Block-collective (every thread calls it; it synchronises the block).
template <int TILE>
__device__ void sched_init(const DecodeParams& p, SchedState& st) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (!p.balanced) {
    if (tid == 0) {
      st.fixed_pending = 1;
      st.U = p.num_kv_heads * p.head_groups;
    }
    __syncthreads();
    return;
  }
  __shared__ long long red[kThreads / 32];
  __shared__ long long found[2];
  const int U = p.num_kv_heads * p.head_groups;
  // Up to kScanCache sequences per thread are kept in registers (thread t holds the
  // sequences [t * kScanCache, (t + 1) * kScanCache)), so that for num_seqs <=
  // kThreads * kScanCache the lengths are read once and one block scan finds the start.
  constexpr int kScanCache = 8;
  const bool cached = p.num_seqs <= kThreads * kScanCache;
  int tl[kScanCache];
  long long part = 0;
  if (cached) {
#pragma unroll
    for (int j = 0; j < kScanCache; ++j) {
      const int sq = tid * kScanCache + j;
      tl[j] = sq < p.num_seqs ? unit_tiles<TILE>(eff_ctx(p, sq)) + p.unit_cost : 0;
      part += tl[j];
    }
  } else {
    for (int sq = tid; sq < p.num_seqs; sq += kThreads)
      part += unit_tiles<TILE>(eff_ctx(p, sq)) + p.unit_cost;
  }
  // inclusive block scan of the per-thread sums (cached layout: sequence order)
  long long x = part;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long v = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += v;
  }
  if (lane == 31) red[warp] = x;
  __syncthreads();
  long long total = 0, before = 0;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) {
    if (i < warp) before += red[i];
    total += red[i];
  }
  const long long excl = before + x - part;  // items before this thread's sequences
  // lanes when U divides the grid with at most 1/32 of it idle
  const long long grid = p.sched_ctas;
  const bool lanes = (long long)U <= grid && (grid - grid / U * U) * 32 <= grid;
  const long long W = lanes ? total : total * U;
  long long G = lanes ? grid / U : grid;
  const long long by_work = W / p.min_tiles;  // every rank gets >= min_tiles items
  if (G > by_work) G = by_work > 0 ? by_work : 1;
  const long long c = blockIdx.x;
  const long long rank = lanes ? c / U : c;
  long long w = 0, w_end = 0;
  if (rank < G) {  // uniform across the block
    w = W * rank / G;
    w_end = W * (rank + 1) / G;
    // the sequence whose tile prefix P(s) satisfies P(s) <= w' < P(s) + tiles(s), with
    // w' = w for lanes and w / U for the unit-major order
    const long long q = lanes ? w : w / U;
    if (cached) {
      if (excl <= q && q < excl + part) {
        long long pre = excl;
#pragma unroll
        for (int j = 0; j < kScanCache; ++j) {
          if (pre <= q && q < pre + tl[j]) {
            found[0] = tid * kScanCache + j;
            found[1] = pre;
          }
          pre += tl[j];
        }
      }
      __syncthreads();
    } else {
      long long carry = 0;
      for (int base = 0; base < p.num_seqs; base += kThreads) {
        const int sq = base + tid;
        const long long t = sq < p.num_seqs ? unit_tiles<TILE>(eff_ctx(p, sq)) + p.unit_cost : 0;
        long long y = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const long long v = __shfl_up_sync(0xffffffffu, y, o);
          if (lane >= o) y += v;
        }
        __syncthreads();  // red is free again
        if (lane == 31) red[warp] = y;
        __syncthreads();
        long long off = carry, chunk = 0;
#pragma unroll
        for (int i = 0; i < kThreads / 32; ++i) {
          if (i < warp) off += red[i];
          chunk += red[i];
        }
        const long long incl = off + y;
        if (sq < p.num_seqs && incl - t <= q && q < incl) {
          found[0] = sq;
          found[1] = incl - t;
        }
        carry += chunk;
        __syncthreads();
        if (carry > q) break;
      }
    }
  }
  if (tid == 0) {
    st.W = W;
    st.G = G;
    st.U = U;
    st.w = w;
    st.w_end = w_end;
    st.lanes = lanes ? 1 : 0;
    st.rank = (int)rank;
    st.fixed_pending = 0;
    if (w < w_end) {
      st.seq = (int)found[0];
      st.eff = eff_ctx(p, st.seq);
      st.nt = unit_tiles<TILE>(st.eff);
      if (lanes) {
        st.y = (int)(c % U);
        st.unit_start = found[1];
      } else {
        const long long r = w - found[1] * U;
        st.y = (int)(r / (st.nt + p.unit_cost));
        st.unit_start = found[1] * U + (long long)st.y * (st.nt + p.unit_cost);
      }
    }
  }
  __syncthreads();
}

// Block-collective: moves st.cur to the CTA's next segment; false when none is left.
// Its first barrier also ends the previous segment's use of shared memory.
template <int TILE>
__device__ bool sched_next(const DecodeParams& p, SchedState& st) {
  __syncthreads();
  if (threadIdx.x == 0) {
    Seg& sg = st.cur;
    int has = 0;
    if (!p.balanced) {
      if (st.fixed_pending) {
        st.fixed_pending = 0;
        const SplitRange rng = split_range(p, blockIdx.z, blockIdx.x);
        if (!(blockIdx.x > 0 && rng.begin >= rng.end)) {
          has = 1;
          sg.seq = blockIdx.z;
          sg.y = blockIdx.y;
          sg.begin = rng.begin;
          sg.end = rng.end;
          sg.nparts = rng.active;
          sg.part = blockIdx.x;
          sg.c_first = sg.first_off = 0;
          sg.cta_base = 0;
          sg.cta_stride = 1;
        }
      }
    } else if (st.w < st.w_end) {
      // A unit's items are unit_cost charge items, then its nt tiles: the charge stands
      // for the fixed cost of a segment, so a rank whose range crosses into a new unit
      // streams that many fewer tiles.
      const int nt = st.nt;
      const long long first = st.unit_start + p.unit_cost;  // item of the unit's tile 0
      const long long tb = st.w > first ? st.w - first : 0;
      const long long rem = st.w_end - first;
      const long long te = rem < nt ? rem : nt;
      if (te <= tb) {
        st.w = st.w_end;  // the range ends inside the unit's charge items
      } else {
        has = 1;
        sg.seq = st.seq;
        sg.y = st.y;
        sg.begin = (int)tb * TILE;
        sg.end = min((int)te * TILE, st.eff);
        const long long c_first = cta_of(st, first);
        const long long c_last = cta_of(st, first + nt - 1);
        sg.nparts = (int)(c_last - c_first + 1);
        sg.part = (int)(st.rank - c_first);
        sg.c_first = (int)c_first;
        sg.first_off = (st.W * c_first / st.G) < st.unit_start ? 1 : 0;
        sg.cta_base = st.lanes ? st.y : 0;
        sg.cta_stride = st.lanes ? st.U : 1;
        st.w = first + te;
        if (te == nt) {
          st.unit_start = first + nt;
          const bool next_seq = st.lanes || ++st.y == st.U;
          if (next_seq) {
            if (!st.lanes) st.y = 0;
            ++st.seq;
            if (st.w < st.w_end) {
              st.eff = eff_ctx(p, st.seq);
              st.nt = unit_tiles<TILE>(st.eff);
            }
          }
        }
      }
    }
    st.has = has;
  }
  __syncthreads();
  return st.has != 0;
}

// Row (of head_dim floats in part_acc, of 2 floats in part_ml) of partial k, head h.
__device__ __forceinline__ int64_t part_row(const DecodeParams& p, const Seg& sg, int h0, int k,
                                            int h) {
  if (p.balanced) {
    const int cta = sg.cta_base + sg.cta_stride * (sg.c_first + k);
    const int slot = 2 * cta + (k == 0 ? sg.first_off : 0);
    return (int64_t)slot * p.heads_per_cta + h;
  }
  return ((int64_t)sg.seq * p.num_heads + h0 + h) * p.num_splits + k;
}

// Block-table slice of the segment in shared memory (validated pages, -1 = none).
struct BlockSlice {
  int lo, n;  // first logical block and count; n > kMaxBtSmem = not staged
};
__device__ __forceinline__ BlockSlice stage_block_table(const DecodeParams& p, int seq,
                                                        const TokRange& rng, int* bt_s,
                                                        bool count) {
  BlockSlice s{0, 0};
  if (rng.end > rng.begin) {
    int hi, off;
    split_token(p, rng.begin, s.lo, off);
    split_token(p, rng.end - 1, hi, off);
    s.n = hi - s.lo + 1;
  }
  if (s.n <= kMaxBtSmem) {
    for (int i = threadIdx.x; i < s.n; i += blockDim.x) bt_s[i] = page_of_block(p, seq, s.lo + i, count);
  } else if (count) {  // not staged: the loads look pages up unchecked-for-counting, so count here
    for (int i = threadIdx.x; i < s.n; i += blockDim.x) page_of_block(p, seq, s.lo + i, true);
  }
  return s;
}
__device__ __forceinline__ int slice_page(const DecodeParams& p, int seq, const BlockSlice& s,
                                          const int* bt_s, int blk) {
  return s.n <= kMaxBtSmem ? bt_s[blk - s.lo] : page_of_block(p, seq, blk, false);
}

// ---------------------------------------------------------------- shared epilogue
// Arrival on a unit's counter: thread 0's release/acquire add at gpu scope, after a
// barrier that orders every thread's partial stores before it (the split-K semaphore
// pattern). The last to arrive then reads the others' partials after a second barrier.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* ctr, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(ctr), "r"(v)
               : "memory");
  return old;
}

// The CTA's result for its nh heads is staged in shared memory: o_s[h * ld + d]
// (unnormalised), m_s[h] (log2 units), l_s[h]. A unit finished by one segment writes
// out = o * v_scale / l directly. Otherwise the segment stores its (m, l, o) partial and
// the last to arrive (per-unit counter) merges all partials in one online pass (running
// maximum with rescaling, the same arithmetic as the softmax) and writes the output; it
// also zeroes the counter for the next launch.
// wbuf (wcap floats of shared memory the CTA no longer needs, or nullptr) holds the
// merge's per-(partial, head) weights. The merge then computes each weight once, one
// warp per head, and its output loop is one independent load and one FMA per partial,
// so a unit split over many CTAs (small batches of long contexts) merges in a few L2
// round trips instead of one per partial.
template <typename QT>
__device__ void finish_cta(const DecodeParams& p, const Seg& sg, int h0, int nh,
                           const float* o_s, int ld, const float* m_s, const float* l_s,
                           float* wbuf = nullptr, int wcap = 0) {
  const int D = p.head_dim;
  const int seq = sg.seq, active = sg.nparts;
  const float vs = p.v_scale != nullptr ? __ldg(p.v_scale) : 1.0f;
  QT* op = reinterpret_cast<QT*>(p.out);
  if (active == 1) {
    for (int idx = threadIdx.x; idx < nh * D; idx += blockDim.x) {
      const int h = idx / D, d = idx - h * D;
      op[(int64_t)seq * p.o_sb + (int64_t)(h0 + h) * p.o_sh + d] =
          from_f32<QT>(o_s[h * ld + d] * vs / l_s[h]);
    }
    return;
  }
  for (int idx = threadIdx.x; idx < nh * D; idx += blockDim.x) {
    const int h = idx / D, d = idx - h * D;
    const int64_t b = part_row(p, sg, h0, sg.part, h);
    __stcg(p.part_acc + b * D + d, o_s[h * ld + d]);
    if (d == 0) {
      __stcg(p.part_ml + b * 2 + 0, m_s[h]);
      __stcg(p.part_ml + b * 2 + 1, l_s[h]);
    }
  }
  __syncthreads();
  __shared__ bool last;
  unsigned int* ctr = p.arrivals + (int64_t)seq * p.num_kv_heads * p.head_groups + sg.y;
  if (threadIdx.x == 0) last = atom_add_acq_rel_gpu(ctr, 1u) == (unsigned)(active - 1);
  __syncthreads();
  if (!last) return;
  constexpr int OUT = 4;
  if (wbuf != nullptr && (active + 1) * nh <= wcap) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    // wbuf[s * nh + h] = exp2(m_s,h - M_h) (0 for a partial without visible tokens);
    // wbuf[active * nh + h] = L_h = sum_s l_s,h * wbuf[s * nh + h]
    for (int h = warp; h < nh; h += nwarps) {
      float mx = -INFINITY;
      for (int s = lane; s < active; s += 32)
        mx = fmaxf(mx, __ldcg(p.part_ml + part_row(p, sg, h0, s, h) * 2));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float l = 0.0f;
      for (int s = lane; s < active; s += 32) {
        const int64_t b = part_row(p, sg, h0, s, h);
        const float m = __ldcg(p.part_ml + b * 2), lv = __ldcg(p.part_ml + b * 2 + 1);
        const float c = m == -INFINITY ? 0.0f : exp2f(m - mx);
        wbuf[s * nh + h] = c;
        l = fmaf(lv, c, l);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0) wbuf[active * nh + h] = l;
    }
    __syncthreads();
    for (int base = threadIdx.x; base < nh * D; base += OUT * blockDim.x) {
      float O[OUT];
      int hh[OUT], dd[OUT];
#pragma unroll
      for (int i = 0; i < OUT; ++i) {
        const int idx = base + i * blockDim.x;
        const bool live = idx < nh * D;
        hh[i] = live ? idx / D : 0;
        dd[i] = live ? idx - hh[i] * D : 0;
        O[i] = 0.0f;
      }
#pragma unroll 8
      for (int s = 0; s < active; ++s)
#pragma unroll
        for (int i = 0; i < OUT; ++i)
          O[i] = fmaf(__ldcg(p.part_acc + part_row(p, sg, h0, s, hh[i]) * D + dd[i]),
                      wbuf[s * nh + hh[i]], O[i]);
#pragma unroll
      for (int i = 0; i < OUT; ++i) {
        const int idx = base + i * blockDim.x;
        if (idx < nh * D)
          op[(int64_t)seq * p.o_sb + (int64_t)(h0 + hh[i]) * p.o_sh + dd[i]] =
              from_f32<QT>(O[i] * vs / wbuf[active * nh + hh[i]]);
      }
    }
    if (threadIdx.x == 0) *ctr = 0u;
    return;
  }
  // Without a weight buffer (CUDA-core kernel): OUT outputs per thread at a time, two
  // passes over the partials: their maximum, then
  // the weighted sums; the loads of up to 8 partials are independent of each other, so
  // they are in flight together instead of one online step after another.
  for (int base = threadIdx.x; base < nh * D; base += OUT * blockDim.x) {
    float M[OUT], L[OUT], O[OUT];
    int64_t row[OUT];
    bool live[OUT];
#pragma unroll
    for (int i = 0; i < OUT; ++i) {
      const int idx = base + i * blockDim.x;
      live[i] = idx < nh * D;
      const int h = live[i] ? idx / D : 0;
      row[i] = (int64_t)h;  // head, turned into the partial row below
      M[i] = -INFINITY, L[i] = 0.0f, O[i] = 0.0f;
    }
#pragma unroll 8
    for (int s = 0; s < active; ++s)
#pragma unroll
      for (int i = 0; i < OUT; ++i)
        if (live[i]) M[i] = fmaxf(M[i], __ldcg(p.part_ml + part_row(p, sg, h0, s, (int)row[i]) * 2));
#pragma unroll 8
    for (int s = 0; s < active; ++s) {
#pragma unroll
      for (int i = 0; i < OUT; ++i) {
        if (!live[i]) continue;
        const int idx = base + i * blockDim.x;
        const int h = (int)row[i], d = idx - h * D;
        const int64_t b = part_row(p, sg, h0, s, h);
        const float m = __ldcg(p.part_ml + b * 2), l = __ldcg(p.part_ml + b * 2 + 1);
        const float a = __ldcg(p.part_acc + b * D + d);
        const float c = m == -INFINITY ? 0.0f : exp2f(m - M[i]);
        O[i] = fmaf(a, c, O[i]);
        L[i] = fmaf(l, c, L[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < OUT; ++i) {
      if (!live[i]) continue;
      const int idx = base + i * blockDim.x;
      const int h = idx / D, d = idx - h * D;
      op[(int64_t)seq * p.o_sb + (int64_t)(h0 + h) * p.o_sh + d] = from_f32<QT>(O[i] * vs / L[i]);
    }
  }
  if (threadIdx.x == 0) *ctr = 0u;
}

// Swizzle key of an e4m3 V row in the FP8-MMA kernel's tiles: bits 0, 1 and 3 of the row
// (rows repeat it every 16). That kernel's transposed 8-bit loads read the rows
// {0,1,8,9,2,3,10,11} (and those + 4) together; their keys are distinct, so each such
// 8-row read touches every bank once.
__device__ __forceinline__ int v_swizzle_key(int row) { return (row & 3) | ((row >> 1) & 4); }

// ---------------------------------------------------------------- tensor-core tile loads
// Issues the cp.async copies of one K/V tile (TILE token rows of ROWB bytes of one kv
// head, starting at token t0) into the stage's buffers, 16-byte chunks XOR-swizzled by
// row (chunk ^ (row & 7)), and writes the stage's per-row valid flags. Rows past the
// segment or on a missing page are zero-filled (src-size 0) and flagged invalid.
// When the tile lies inside one page (power-of-two block_size >= TILE) the thread's
// rows are one base address plus a constant stride, so a full tile costs two cp.async
// and one address add per pass.
template <int TILE, int ROWB, bool kVKey = false>
__device__ __forceinline__ void load_kv_tile(const DecodeParams& p, int seq,
                                             const BlockSlice& slice, const int* bt_s,
                                             const TokRange& rng, int t0, uint8_t* kd,
                                             uint8_t* vd, uint8_t* valid, int64_t row_stride,
                                             int64_t head_off, bool one_page_per_tile,
                                             float* rs = nullptr, int kvh = 0) {
  constexpr int CPR = ROWB / 16;         // 16-byte chunks per row
  constexpr int RPP = kThreads / CPR;    // rows per pass (a multiple of 8)
  constexpr int PASSES = TILE / RPP;
  static_assert(RPP % 8 == 0 && TILE % RPP == 0 && TILE <= kThreads, "tile geometry");
  const int tid = threadIdx.x, ld_c = tid % CPR, ld_r0 = tid / CPR;
  // (r & 7) is the same for all of this thread's rows r = ld_r0 + i * RPP
  const uint32_t soff0 = ld_r0 * ROWB + ((ld_c ^ (ld_r0 & 7)) << 4);
  const uint32_t kd0 = smem_u32(kd) + soff0;
  const uint32_t vd0 =
      smem_u32(vd) + (kVKey ? ld_r0 * ROWB + ((ld_c ^ v_swizzle_key(ld_r0)) << 4) : soff0);
  // per-token scales of 8-bit pages: entry r < TILE is row r's K scale, TILE + r its V
  // scale (zero for rows that are not loaded)
  if (rs != nullptr && one_page_per_tile) {  // one page: row r's scales are r * KVH apart
    static_assert(TILE == kThreads || 2 * TILE == kThreads, "one K or V row scale pair per thread");
    const int page = slice_page(p, seq, slice, bt_s, t0 >> p.bs_shift);
    const int nrows = page >= 0 ? min(TILE, rng.end - t0) : 0;
    const int64_t base =
        ((int64_t)(page >= 0 ? page : 0) * p.block_size + (t0 & ((1 << p.bs_shift) - 1))) * p.num_kv_heads + kvh;
    if constexpr (TILE == kThreads) {  // row tid: its K scale and its V scale
      const int64_t off = base + (int64_t)tid * p.num_kv_heads;
      const bool ok = tid < nrows;
      cp_async_4(smem_u32(rs + tid), ok ? p.k_scales + off : p.k_scales, ok ? 4 : 0);
      cp_async_4(smem_u32(rs + TILE + tid), ok ? p.v_scales + off : p.v_scales, ok ? 4 : 0);
    } else {  // threads [0, TILE): K scales; [TILE, 2 TILE): V scales (whole warps each)
      const int r = tid < TILE ? tid : tid - TILE;
      const float* src = (tid < TILE ? p.k_scales : p.v_scales);
      const bool ok = r < nrows;
      cp_async_4(smem_u32(rs + tid), ok ? src + base + (int64_t)r * p.num_kv_heads : src, ok ? 4 : 0);
    }
  } else if (rs != nullptr) {
    for (int i = tid; i < 2 * TILE; i += kThreads) {
      const int r = i < TILE ? i : i - TILE;
      const float* src = i < TILE ? p.k_scales : p.v_scales;
      const int t = t0 + r;
      int page = -1, boff = 0;
      if (t < rng.end) {
        int blk;
        split_token(p, t, blk, boff);
        page = slice_page(p, seq, slice, bt_s, blk);
      }
      const int64_t idx = page >= 0 ? ((int64_t)page * p.block_size + boff) * p.num_kv_heads + kvh : 0;
      cp_async_4(smem_u32(rs + i), src + idx, page >= 0 ? 4 : 0);
    }
  }
  if (one_page_per_tile) {
    const int page = slice_page(p, seq, slice, bt_s, t0 >> p.bs_shift);
    const int nrows = page >= 0 ? min(TILE, rng.end - t0) : 0;
    const int64_t base =
        page >= 0 ? ((int64_t)page * p.block_size + (t0 & ((1 << p.bs_shift) - 1)) + ld_r0) *
                            row_stride + head_off + ld_c * 16
                  : 0;
    const uint8_t* kp = p.k_cache + base;
    const uint8_t* vp = p.v_cache + base;
    const int64_t step = (int64_t)RPP * row_stride;
    if (nrows == TILE) {
#pragma unroll
      for (int i = 0; i < PASSES; ++i) {
        cp_async_16(kd0 + i * RPP * ROWB, kp + i * step, 16);
        cp_async_16(vd0 + i * RPP * ROWB, vp + i * step, 16);
      }
    } else {
#pragma unroll
      for (int i = 0; i < PASSES; ++i) {
        const bool ok = ld_r0 + i * RPP < nrows;
        cp_async_16(kd0 + i * RPP * ROWB, ok ? kp + i * step : p.k_cache, ok ? 16 : 0);
        cp_async_16(vd0 + i * RPP * ROWB, ok ? vp + i * step : p.v_cache, ok ? 16 : 0);
      }
    }
    if (tid < TILE) valid[tid] = tid < nrows ? 1 : 0;
    return;
  }
#pragma unroll
  for (int i = 0; i < PASSES; ++i) {
    const int r = ld_r0 + i * RPP;
    const int t = t0 + r;
    int page = -1, boff = 0;
    if (t < rng.end) {
      int blk;
      split_token(p, t, blk, boff);
      page = slice_page(p, seq, slice, bt_s, blk);
    }
    const bool ok = page >= 0;
    const int64_t off =
        ok ? ((int64_t)page * p.block_size + boff) * row_stride + head_off + ld_c * 16 : 0;
    cp_async_16(kd0 + i * RPP * ROWB, p.k_cache + off, ok ? 16 : 0);
    cp_async_16(vd0 + i * RPP * ROWB, p.v_cache + off, ok ? 16 : 0);
    if (ld_c == 0) valid[r] = ok ? 1 : 0;
  }
}

// The nh query rows (seq, h0 .. h0 + nh - 1) of a segment into q_s (pitch kTcD elements):
// 16-byte cp.async chunks when the rows are 16-byte aligned (joining the caller's next
// cp.async group), else element copies.
template <typename QT>
__device__ __forceinline__ void load_q_rows(const DecodeParams& p, int seq, int h0, int nh,
                                            QT* q_s) {
  constexpr int D = kTcD;
  constexpr int PER = 16 / (int)sizeof(QT);  // elements per 16-byte chunk
  constexpr int CPR = D / PER;
  const QT* qp = reinterpret_cast<const QT*>(p.q) + (int64_t)seq * p.q_sb + (int64_t)h0 * p.q_sh;
  if (p.q_vec16) {
    for (int c = threadIdx.x; c < nh * CPR; c += kThreads) {
      const int r = c / CPR, k = c - r * CPR;
      cp_async_16(smem_u32(q_s + r * D + k * PER), qp + (int64_t)r * p.q_sh + k * PER, 16);
    }
  } else {
    for (int i = threadIdx.x; i < nh * D; i += kThreads) {
      const int r = i / D, d = i - r * D;
      q_s[r * D + d] = qp[(int64_t)r * p.q_sh + d];
    }
  }
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
  constexpr bool kByte = sizeof(CT) == 1;  // e4m3 or int8 pages
  constexpr int kPer = 16 / EB;  // elements per 16-byte chunk
  const int D = p.head_dim;
  const int row_bytes = D * EB;
  const int row_pitch = row_bytes + 16;  // padding keeps lane-per-row reads conflict-free
  const int chunks = row_bytes / 16;
  const int ring = 4 * kGenTile * row_pitch;
  const int epi = kMaxHeadsPerCta * D * 4;

  uint8_t* kbuf = smem;                                             // [2][kGenTile][row_pitch]
  uint8_t* vbuf = kbuf + 2 * kGenTile * row_pitch;                  // [2][kGenTile][row_pitch]
  float* q_s = reinterpret_cast<float*>(smem + (ring > epi ? ring : epi));  // [16][D]
  float* s_s = q_s + kMaxHeadsPerCta * D;                          // [16][kGenTile]
  float* m_s = s_s + kMaxHeadsPerCta * kGenTile;                   // [16]
  float* l_s = m_s + kMaxHeadsPerCta;                              // [16]
  float* a_s = l_s + kMaxHeadsPerCta;                              // [16]
  uint8_t* valid = reinterpret_cast<uint8_t*>(a_s + kMaxHeadsPerCta);  // [2][kGenTile]
  int* bt_s = reinterpret_cast<int*>(valid + 2 * kGenTile);        // [kMaxBtSmem]
  float* rs_s = reinterpret_cast<float*>(bt_s + kMaxBtSmem);       // [2][2][kGenTile] row scales
  const bool per_token = p.k_scales != nullptr;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ SchedState sched;
  sched_init<kGenTile>(p, sched);
  pdl_wait();  // pages may have been written by the kernel this launch overlaps
  while (sched_next<kGenTile>(p, sched)) {
  const TokRange rng{sched.cur.begin, sched.cur.end};
  const int seq = sched.cur.seq;
  const int kvh = sched.cur.y / p.head_groups;
  const int hg = sched.cur.y - kvh * p.head_groups;
  const int h0 = kvh * p.group + hg * p.heads_per_cta;
  const int nh = min(p.heads_per_cta, p.group - hg * p.heads_per_cta);
  const bool count_invalid = (kvh == 0 && hg == 0);

  const BlockSlice slice = stage_block_table(p, seq, rng, bt_s, count_invalid);

  const float ks = (kByte && !per_token) ? __ldg(p.k_scale) : 1.0f;
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
  __syncthreads();

  const int64_t row_stride = (int64_t)p.num_kv_heads * row_bytes;  // bytes between tokens
  const int64_t head_off = (int64_t)kvh * row_bytes;
  auto load_tile = [&](int t0, int stage) {
    uint8_t* kd = kbuf + stage * kGenTile * row_pitch;
    uint8_t* vd = vbuf + stage * kGenTile * row_pitch;
    for (int idx = tid; idx < kGenTile * chunks; idx += kThreads) {
      const int r = idx / chunks, c = idx - r * chunks;
      const int t = t0 + r;
      int page = -1, boff = 0;
      if (t < rng.end) {
        int blk;
        split_token(p, t, blk, boff);
        page = slice_page(p, seq, slice, bt_s, blk);
      }
      const bool ok = page >= 0;
      const int64_t off =
          ok ? ((int64_t)page * p.block_size + boff) * row_stride + head_off + c * 16 : 0;
      cp_async_16(smem_u32(kd + r * row_pitch + c * 16), p.k_cache + off, ok ? 16 : 0);
      cp_async_16(smem_u32(vd + r * row_pitch + c * 16), p.v_cache + off, ok ? 16 : 0);
      if (c == 0) {
        valid[stage * kGenTile + r] = ok ? 1 : 0;
        if (per_token) {
          const int64_t si = ok ? ((int64_t)page * p.block_size + boff) * p.num_kv_heads + kvh : 0;
          float* rs = rs_s + stage * 2 * kGenTile;
          cp_async_4(smem_u32(rs + r), p.k_scales + si, ok ? 4 : 0);
          cp_async_4(smem_u32(rs + kGenTile + r), p.v_scales + si, ok ? 4 : 0);
        }
      }
    }
  };

  constexpr int kMaxDpt = 2;  // head_dim <= 256 = 2 columns per thread
  float acc[kMaxHeadsPerCta][kMaxDpt];
#pragma unroll
  for (int h = 0; h < kMaxHeadsPerCta; ++h)
#pragma unroll
    for (int j = 0; j < kMaxDpt; ++j) acc[h][j] = 0.0f;

  const int span = rng.end > rng.begin ? rng.end - rng.begin : 0;
  const int ntiles = (span + kGenTile - 1) / kGenTile;
  if (ntiles > 0) load_tile(rng.begin, 0);
  cp_async_commit();
  for (int it = 0; it < ntiles; ++it) {
    const int stage = it & 1;
    if (it + 1 < ntiles) load_tile(rng.begin + (it + 1) * kGenTile, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint8_t* kt = kbuf + stage * kGenTile * row_pitch;
    const uint8_t* vt = vbuf + stage * kGenTile * row_pitch;
    const uint8_t* vld = valid + stage * kGenTile;
    const float* rs = rs_s + stage * 2 * kGenTile;  // row scales (per_token only)

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
      if (per_token) s *= rs[lane];
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
          float v = to_f32(reinterpret_cast<const CT*>(vt + r * row_pitch)[d]);
          if (per_token) v *= rs[kGenTile + r];
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

  // stage the result in the (now idle) ring and finish
  float* o_s = reinterpret_cast<float*>(smem);  // [16][D]
#pragma unroll
  for (int j = 0; j < kMaxDpt; ++j) {
    const int d = tid + j * kThreads;
    if (d < D) {
#pragma unroll
      for (int h = 0; h < kMaxHeadsPerCta; ++h)
        if (h < nh) o_s[h * D + d] = acc[h][j];
    }
  }
  __syncthreads();
  finish_cta<QT>(p, sched.cur, h0, nh, o_s, D, m_s, l_s);
  }
}

size_t generic_smem_bytes(int head_dim, int elem_bytes) {
  const int row_pitch = head_dim * elem_bytes + 16;
  const size_t ring = (size_t)4 * kGenTile * row_pitch;
  const size_t epi = (size_t)kMaxHeadsPerCta * head_dim * 4;
  return (ring > epi ? ring : epi) + (size_t)kMaxHeadsPerCta * head_dim * 4 +
         (size_t)kMaxHeadsPerCta * kGenTile * 4 + 3 * kMaxHeadsPerCta * 4 + 2 * kGenTile +
         kMaxBtSmem * 4 + 2 * 2 * kGenTile * 4;
}

// ============================================================ tensor-core kernel
// head_dim = 128; query bf16 with bf16 pages, f16 with f16 pages, or bf16/f16 with
// int8 pages (f16 MMAs). NT = query heads of the CTA in units of 8 (MMA N tiles).
// MMA operand type of a page type; int8 pages are converted to f16 in registers, two
// elements per conversion (e4m3 pages take the FP8-MMA kernel below).
template <typename CT> struct TcTraits;
template <> struct TcTraits<bf16> {
  using MT = bf16;
  static constexpr bool kByte = false;
  // 16-bit pages feed the MMA as they are; the 8-bit branch that calls this is dead
  static __device__ __forceinline__ uint32_t to_f16x2(uint16_t) { return 0u; }
};
template <> struct TcTraits<f16> {
  using MT = f16;
  static constexpr bool kByte = false;
  // 16-bit pages feed the MMA as they are; the 8-bit branch that calls this is dead
  static __device__ __forceinline__ uint32_t to_f16x2(uint16_t) { return 0u; }
};
// int8 pages enter the f16 MMAs as x + kInt8Bias (exact in f16), and the kernel takes the
// bias back out of S and O.
constexpr float kInt8Bias = 1152.0f;
template <> struct TcTraits<int8_t> {
  using MT = f16;
  static constexpr bool kByte = true;
  static __device__ __forceinline__ uint32_t to_f16x2(uint16_t v) { return s8x2_to_f16x2(v); }
};


__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

// Epilogue buffers (floats), for a CTA of up to 8*NT query heads: the 4 warps' partial
// O^T [4][8NT][D+4] (warp 0's slot is overwritten in place by the merged O), their m
// and l [4][8NT] each, the merged m and l [8NT] each.
template <int NT>
constexpr size_t tc_epilogue_bytes() {
  return (size_t)(4 * 8 * NT * (kTcD + 4) + 8 * 8 * NT + 2 * 8 * NT) * 4;
}

template <typename CT, int NT, int STAGES>
constexpr size_t tc_front_bytes() {  // ring, reused by the epilogue
  constexpr size_t ring = (size_t)STAGES * 2 * kTcTile * kTcD * sizeof(CT);
  return ring > tc_epilogue_bytes<NT>() ? ring : tc_epilogue_bytes<NT>();
}
template <typename CT, int NT, int STAGES>
constexpr size_t tc_smem_bytes() {  // + valid flags + block table + query rows + row scales
  return tc_front_bytes<CT, NT, STAGES>() + (size_t)STAGES * kTcTile + kMaxBtSmem * 4 +
         (size_t)8 * NT * kTcD * 2 + (size_t)STAGES * 2 * kTcTile * 4;
}

// kPT: 8-bit pages with a scale per (page, row, kv head): S^T rows are multiplied by
// the K scale of their token and P by the V scale before the PV product (the softmax
// denominator uses the unscaled P).
template <typename QT, typename CT, int NT, int STAGES, int MINB, bool kPT>
__global__ void __launch_bounds__(kThreads, MINB)
paged_decode_tc_kernel(const DecodeParams p) {
  using Tr = TcTraits<CT>;
  using MT = typename Tr::MT;
  constexpr bool kFp8 = Tr::kByte;  // 8-bit pages (e4m3 or int8), converted to f16
  constexpr bool kBias = std::is_same<CT, int8_t>::value;  // int8 pages as x + 1152 (below)
  constexpr int D = kTcD;
  constexpr int EB = sizeof(CT);
  constexpr int ROWB = D * EB;    // 256 (16-bit) or 128 (e4m3) bytes per token row
  constexpr int TILE_BYTES = kTcTile * ROWB;
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  constexpr size_t FRONT = tc_front_bytes<CT, NT, STAGES>();

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* valid = smem + FRONT;                                 // [STAGES][kTcTile]
  int* bt_s = reinterpret_cast<int*>(valid + STAGES * kTcTile);  // [kMaxBtSmem]
  QT* q_s = reinterpret_cast<QT*>(bt_s + kMaxBtSmem);             // [8 * NT][D]
  float* rs_s = reinterpret_cast<float*>(q_s + 8 * NT * D);       // [STAGES][2][kTcTile]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  // Segment hand-over: when the epilogue fits in one ring stage, the next segment's first
  // tiles are issued into the free stages before this segment's epilogue runs in the
  // stage of its last tile, so the page fetch overlaps the merge and the partial write.
  // Ring stage of tile `it` of a segment: (gt + it) % STAGES, gt = tiles begun before it.
  constexpr bool kPrefetch = tc_epilogue_bytes<NT>() <= (size_t)STAGE_BYTES;
  const int64_t row_stride = (int64_t)p.num_kv_heads * ROWB;
  // A tile never straddles a page when block_size is a power of two >= the tile.
  const bool one_page_per_tile = p.bs_shift >= 6;
  __shared__ SchedState sched;
  sched_init<kTcTile>(p, sched);
  bool has = sched_next<kTcTile>(p, sched);
  bool prefetched = false;
  int gt = 0;
  BlockSlice slice{0, 0};
  while (has) {
  const TokRange rng{sched.cur.begin, sched.cur.end};
  const int seq = sched.cur.seq;
  const int kvh = sched.cur.y / p.head_groups;
  const int hgrp = sched.cur.y - kvh * p.head_groups;
  const int h0 = kvh * p.group + hgrp * p.heads_per_cta;
  const int nh = min(p.heads_per_cta, p.group - hgrp * p.heads_per_cta);
  const bool count_invalid = (kvh == 0 && hgrp == 0);

  const int ntiles = (rng.end - rng.begin + kTcTile - 1) / kTcTile;  // 0 when empty
  if (!prefetched) {
    slice = stage_block_table(p, seq, rng, bt_s, count_invalid);
    __syncthreads();
  }

  // ---- producer: all threads issue 16-byte cp.async for their rows/chunks
  const int64_t head_off = (int64_t)kvh * ROWB;
  auto load_tile = [&](int it) {
    const int stage = (gt + it) % STAGES;
    uint8_t* kd = smem + stage * STAGE_BYTES;
    load_kv_tile<kTcTile, ROWB>(p, seq, slice, bt_s, rng, rng.begin + it * kTcTile, kd,
                                kd + TILE_BYTES, valid + stage * kTcTile, row_stride, head_off,
                                one_page_per_tile, kPT ? rs_s + stage * 2 * kTcTile : nullptr, kvh);
  };

  // prologue: the query rows, then STAGES-1 tiles, in flight before the query fragments
  if (!prefetched) {
    load_q_rows<QT>(p, seq, h0, nh, q_s);
    cp_async_commit();
    // Everything above (schedule scan, block-table slice, query rows) may overlap the
    // previous kernel of a programmatic launch; the pages it may have written are read
    // only after it has completed.
    pdl_wait();
#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
      if (s < ntiles) load_tile(s);
      cp_async_commit();
    }
  }

  // ---- Q^T fragments (B operand: K = head_dim, N = query heads of this CTA)
  cp_async_wait<STAGES - 1>();  // the query rows' group (older than the tiles')
  __syncthreads();
  auto qval = [&](int row, int d) -> float { return row < nh ? to_f32(q_s[row * D + d]) : 0.0f; };
  // head_dim index of B-fragment element (k-step ks, register half, element e).
  // 16-bit pages: b0 = k 2tig,2tig+1; b1 = k 2tig+8,2tig+9 (PTX m16n8k16 layout).
  // e4m3 pages: k is permuted so that one ldmatrix word (the 4 bytes d = 4tig..4tig+3)
  // feeds both A registers of a k-step; Q uses the same permutation.
  auto qcol = [&](int ks, int half, int e) -> int {
    if (kFp8) return 16 * ks + 4 * tig + 2 * half + e;
    return 16 * ks + 8 * half + 2 * tig + e;
  };
  float qpow2 = 1.0f;  // FP8 path: bf16 query rescaled by a power of two into f16 range
  if (kFp8 && std::is_same<QT, bf16>::value) {
    float mx = 0.0f;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int e = 0; e < 2; ++e) mx = fmaxf(mx, fabsf(qval(nt * 8 + g, qcol(ks, half, e))));
    mx = warp_max(mx);
    if (mx > 0.0f && isfinite(mx)) {
      int ex;
      frexpf(mx, &ex);                // mx = f * 2^ex, f in [0.5, 1)
      qpow2 = ldexpf(1.0f, 15 - ex);  // max |q| * qpow2 < 2^15 < f16 max
    }
  }
  uint32_t qb[NT][D / 16][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int row = nt * 8 + g;
      qb[nt][ks][0] = pack2<MT>(qval(row, qcol(ks, 0, 0)) * qpow2, qval(row, qcol(ks, 0, 1)) * qpow2);
      qb[nt][ks][1] = pack2<MT>(qval(row, qcol(ks, 1, 0)) * qpow2, qval(row, qcol(ks, 1, 1)) * qpow2);
    }
  // int8 pages enter the MMAs as the exact f16 values x + 1152 (bit pattern 0x64XX with
  // XX = x ^ 0x80), so S^T = K Q^T comes out as S + 1152 * sum_d q[h][d]. qbias holds that
  // offset for heads 2tig + e, from the f16 query values the MMAs use.
  float qbias[NT][2];
  if (kBias) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float sq = 0.0f;  // head g over this lane's k subset
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint32_t w = qb[nt][ks][r];
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
          sq += f.x + f.y;
        }
      sq += __shfl_xor_sync(0xffffffffu, sq, 1);
      sq += __shfl_xor_sync(0xffffffffu, sq, 2);
#pragma unroll
      for (int e = 0; e < 2; ++e)
        qbias[nt][e] = kInt8Bias * __shfl_sync(0xffffffffu, sq, (2 * tig + e) * 4);
    }
  }
  const float ksc = (kFp8 && !kPT) ? __ldg(p.k_scale) : 1.0f;
  const float sc = p.qk_scale_log2 * ksc / qpow2;

  // ---- per-warp softmax state for heads nt*8 + 2tig + e, and O^T accumulators
  float m_run[NT][2], l_run[NT][2];
  float w_run[NT][2];  // int8 pages: sum of the f16 P^T values fed to the PV MMAs, per head
  float o[NT][D / 16][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt][0] = m_run[nt][1] = -INFINITY;
    l_run[nt][0] = l_run[nt][1] = 0.0f;
    w_run[nt][0] = w_run[nt][1] = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 16; ++j) o[nt][j][0] = o[nt][j][1] = o[nt][j][2] = o[nt][j][3] = 0.0f;
  }

  const int lrow = lane & 7;   // ldmatrix: row within the 8x8 matrix this lane addresses
  const int lmat = lane >> 3;  // ldmatrix: which of the 4 matrices
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (it + STAGES - 1 < ntiles) load_tile(it + STAGES - 1);
    cp_async_commit();

    const int stage = (gt + it) % STAGES;
    const uint32_t kbase = smem_u32(smem + stage * STAGE_BYTES);
    const uint32_t vbase = kbase + TILE_BYTES;
    const uint8_t* vld = valid + stage * kTcTile;

    // ---- S^T = K Q^T: this warp's 16 tokens (M) x query heads (N)
    float s[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
    {
      // matrices: 0 = tokens 0-7, 1 = tokens 8-15 (same chunk); 2/3 = next chunk
      const int r = warp * 16 + ((lmat & 1) << 3) + lrow;
      if (!kFp8) {
        // two independent accumulator chains (even / odd k-steps) halve the MMA
        // dependency depth; summed after the loop
        float s2[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) s2[nt][0] = s2[nt][1] = s2[nt][2] = s2[nt][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int lc = 2 * ks + (lmat >> 1);
          uint32_t a[4];
          ldmatrix_x4(kbase + r * ROWB + ((lc ^ lrow) << 4), a[0], a[1], a[2], a[3]);
          // a[0]: tokens 0-7, k 0-7; a[1]: tokens 8-15, k 0-7; a[2]/a[3]: k 8-15
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            Mma<MT>::run((ks & 1) ? s2[nt] : s[nt], a, qb[nt][ks][0], qb[nt][ks][1]);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) s[nt][i] += s2[nt][i];
      } else {
#pragma unroll
        for (int kq = 0; kq < D / 32; ++kq) {
          const int lc = 2 * kq + (lmat >> 1);
          uint32_t x[4];
          ldmatrix_x4(kbase + r * ROWB + ((lc ^ lrow) << 4), x[0], x[1], x[2], x[3]);
#pragma unroll
          for (int hc = 0; hc < 2; ++hc) {
            uint32_t a[4];
            if (kBias) {  // bytes 0,1 / 2,3 -> f16x2 of x + 1152
              const uint32_t xa = x[2 * hc] ^ 0x80808080u, xb = x[2 * hc + 1] ^ 0x80808080u;
              a[0] = __byte_perm(xa, 0x64646464u, 0x5140);
              a[1] = __byte_perm(xb, 0x64646464u, 0x5140);
              a[2] = __byte_perm(xa, 0x64646464u, 0x5342);
              a[3] = __byte_perm(xb, 0x64646464u, 0x5342);
            } else {
              a[0] = Tr::to_f16x2((uint16_t)(x[2 * hc] & 0xffffu));
              a[1] = Tr::to_f16x2((uint16_t)(x[2 * hc + 1] & 0xffffu));
              a[2] = Tr::to_f16x2((uint16_t)(x[2 * hc] >> 16));
              a[3] = Tr::to_f16x2((uint16_t)(x[2 * hc + 1] >> 16));
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
              Mma<MT>::run(s[nt], a, qb[nt][2 * kq + hc][0], qb[nt][2 * kq + hc][1]);
          }
        }
      }
    }

    // ---- int8 pages: take out the +1152 bias's contribution to S^T
    if (kBias) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        s[nt][0] -= qbias[nt][0];
        s[nt][1] -= qbias[nt][1];
        s[nt][2] -= qbias[nt][0];
        s[nt][3] -= qbias[nt][1];
      }
    }
    // Score multiplier per token of this thread (kPT: the token's K scale folded in) and
    // an additive -inf for rows that were not loaded, so a score costs one FFMA (those
    // rows' K bytes and scales are zero-filled: 0 * c - inf = -inf).
    float vsc0 = 1.0f, vsc1 = 1.0f;
    float c0 = sc, c1 = sc;
    if (kPT) {
      const float* rs = rs_s + stage * 2 * kTcTile;
      c0 = sc * rs[warp * 16 + g];
      c1 = sc * rs[warp * 16 + g + 8];
      vsc0 = rs[kTcTile + warp * 16 + g];
      vsc1 = rs[kTcTile + warp * 16 + g + 8];
    }
    const float bias0 = vld[warp * 16 + g] != 0 ? 0.0f : -INFINITY;
    const float bias1 = vld[warp * 16 + g + 8] != 0 ? 0.0f : -INFINITY;

    // ---- online softmax per query head (column of S^T), exp2 domain
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float alpha[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float x0 = fmaf(s[nt][e], c0, bias0);      // token g
        const float x1 = fmaf(s[nt][e + 2], c1, bias1);  // token g + 8
        float mx = fmaxf(x0, x1);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run[nt][e], mx);
        const float base = m_new == -INFINITY ? 0.0f : m_new;
        alpha[e] = exp2f(m_run[nt][e] - base);
        m_run[nt][e] = m_new;
        const float p0 = ex2_approx(x0 - base), p1 = ex2_approx(x1 - base);  // 2^-inf = +0
        l_run[nt][e] = fmaf(l_run[nt][e], alpha[e], p0 + p1);
        s[nt][e] = p0;
        s[nt][e + 2] = p1;
      }
      if (alpha[0] != 1.0f || alpha[1] != 1.0f) {
        const uint64_t a2 = f2_pack(alpha[0], alpha[1]);  // accumulator pairs: heads 2tig, 2tig + 1
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
          f2_unpack(f2_mul(f2_pack(o[nt][j][0], o[nt][j][1]), a2), o[nt][j][0], o[nt][j][1]);
          f2_unpack(f2_mul(f2_pack(o[nt][j][2], o[nt][j][3]), a2), o[nt][j][2], o[nt][j][3]);
        }
      }
      // P^T as the B operand (K = tokens, N = heads): transpose the 8x8 blocks
      const uint32_t u0 = pack2<MT>(s[nt][0] * vsc0, s[nt][1] * vsc0);  // token g, heads 2tig(+1)
      const uint32_t u1 = pack2<MT>(s[nt][2] * vsc1, s[nt][3] * vsc1);  // token g + 8
      if (kBias) {
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u0));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u1));
        w_run[nt][0] = fmaf(w_run[nt][0], alpha[0], f0.x + f1.x);
        w_run[nt][1] = fmaf(w_run[nt][1], alpha[1], f0.y + f1.y);
      }
      pb[nt][0] = movmatrix_trans(u0);  // tokens 0-7
      pb[nt][1] = movmatrix_trans(u1);  // tokens 8-15
    }

    // ---- O^T += V^T P^T, one 16-row (head_dim) M tile per MMA
    if (!kFp8) {
      // matrices: 0 = (tokens 0-7, chunk 2c), 1 = (tokens 0-7, chunk 2c+1),
      //           2 = (tokens 8-15, chunk 2c), 3 = (tokens 8-15, chunk 2c+1)
      const int r = warp * 16 + ((lmat >> 1) << 3) + lrow;
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        const int lc = 2 * c + (lmat & 1);
        uint32_t a[4];
        ldmatrix_x4_trans(vbase + r * ROWB + ((lc ^ lrow) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<MT>::run(o[nt][c], a, pb[nt][0], pb[nt][1]);
      }
    } else {
      // ldmatrix.trans over e4m3 rows: a register holds tokens (2tig, 2tig+1) x
      // d (2g, 2g+1) of a 16-column chunk; a byte permute separates even d (M rows
      // 0-7 of the tile) from odd d (M rows 8-15).
      const int r = warp * 16 + ((lmat & 1) << 3) + lrow;
#pragma unroll
      for (int cq = 0; cq < D / 32; ++cq) {
        const int lc = 2 * cq + (lmat >> 1);
        uint32_t x[4];
        ldmatrix_x4_trans(vbase + r * ROWB + ((lc ^ lrow) << 4), x[0], x[1], x[2], x[3]);
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          uint32_t a[4];
          if (kBias) {  // the same byte order as below, straight to f16x2 of x + 1152
            const uint32_t xa = x[2 * hc] ^ 0x80808080u, xb = x[2 * hc + 1] ^ 0x80808080u;
            a[0] = __byte_perm(xa, 0x64646464u, 0x5240);
            a[1] = __byte_perm(xa, 0x64646464u, 0x5341);
            a[2] = __byte_perm(xb, 0x64646464u, 0x5240);
            a[3] = __byte_perm(xb, 0x64646464u, 0x5341);
          } else {
            const uint32_t ya = __byte_perm(x[2 * hc], 0u, 0x3120);      // tokens 0-7
            const uint32_t yb = __byte_perm(x[2 * hc + 1], 0u, 0x3120);  // tokens 8-15
            a[0] = Tr::to_f16x2((uint16_t)(ya & 0xffffu));
            a[1] = Tr::to_f16x2((uint16_t)(ya >> 16));
            a[2] = Tr::to_f16x2((uint16_t)(yb & 0xffffu));
            a[3] = Tr::to_f16x2((uint16_t)(yb >> 16));
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Mma<MT>::run(o[nt][2 * cq + hc], a, pb[nt][0], pb[nt][1]);
        }
      }
    }
  }
  gt += ntiles;

  // ---- hand over to the next segment, then merge this one
  const Seg done = sched.cur;
  uint8_t* scratch = smem;
  if (kPrefetch) {
    has = sched_next<kTcTile>(p, sched);  // its barrier: every warp is done with the ring
    prefetched = false;
    if (has) {
      const TokRange nr{sched.cur.begin, sched.cur.end};
      const int nkvh = sched.cur.y / p.head_groups;
      const int nhg = sched.cur.y - nkvh * p.head_groups;
      const int nt2 = (nr.end - nr.begin + kTcTile - 1) / kTcTile;
      slice = stage_block_table(p, sched.cur.seq, nr, bt_s, nkvh == 0 && nhg == 0);
      __syncthreads();
      load_q_rows<QT>(p, sched.cur.seq, nkvh * p.group + nhg * p.heads_per_cta,
                      min(p.heads_per_cta, p.group - nhg * p.heads_per_cta), q_s);
      cp_async_commit();
#pragma unroll
      for (int s = 0; s < STAGES - 1; ++s) {
        if (s < nt2) {
          uint8_t* kd = smem + ((gt + s) % STAGES) * STAGE_BYTES;
          load_kv_tile<kTcTile, ROWB>(p, sched.cur.seq, slice, bt_s, nr, nr.begin + s * kTcTile,
                                      kd, kd + TILE_BYTES, valid + ((gt + s) % STAGES) * kTcTile,
                                      row_stride, (int64_t)nkvh * ROWB, one_page_per_tile,
                                      kPT ? rs_s + ((gt + s) % STAGES) * 2 * kTcTile : nullptr,
                                      nkvh);
        }
        cp_async_commit();
      }
      prefetched = true;
    }
    scratch = smem + ((gt + STAGES - 1) % STAGES) * STAGE_BYTES;  // stage of the last tile
  } else {
    cp_async_wait<0>();
    __syncthreads();
  }

  // ---- merge the 4 warps' states through shared memory (in a free ring stage)
  constexpr int RP = D + 4;     // padded row pitch (floats)
  constexpr int HC = 8 * NT;    // head slots of this CTA
  float* red_acc = reinterpret_cast<float*>(scratch);  // [4][HC][RP]; slot 0 becomes the merged O
  float* red_m = red_acc + 4 * HC * RP;             // [4][HC]
  float* red_l = red_m + 4 * HC;                    // [4][HC]
  float* m_s = red_l + 4 * HC;                      // [HC]
  float* l_s = m_s + HC;                            // [HC]
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = l_run[nt][e];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      const int head = nt * 8 + 2 * tig + e;
      float* ra = red_acc + (warp * HC + head) * RP;
      float obias = 0.0f;  // int8 pages: O^T came out as O + 1152 * (sum of P^T values)
      if (kBias) {
        float wsum = w_run[nt][e];
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 4);
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 8);
        wsum += __shfl_xor_sync(0xffffffffu, wsum, 16);
        obias = kInt8Bias * wsum;
      }
#pragma unroll
      for (int j = 0; j < D / 16; ++j) {
        // O^T rows: 16-bit pages d = 16j + g / 16j + 8 + g; e4m3 pages d = 16j + 2g / + 1
        const int d0 = kFp8 ? 16 * j + 2 * g : 16 * j + g;
        const int d1 = kFp8 ? d0 + 1 : d0 + 8;
        ra[d0] = o[nt][j][e] - obias;
        ra[d1] = o[nt][j][e + 2] - obias;
      }
      if (g == 0) {
        red_m[warp * HC + head] = m_run[nt][e];
        red_l[warp * HC + head] = l;
      }
    }
  __syncthreads();
  if (tid < nh) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red_m[w * HC + tid]);
    const float base = M == -INFINITY ? 0.0f : M;
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) L = fmaf(exp2f(red_m[w * HC + tid] - base), red_l[w * HC + tid], L);
    m_s[tid] = M;
    l_s[tid] = L;
  }
  __syncthreads();
  for (int idx = tid; idx < nh * D; idx += kThreads) {
    const int h = idx / D, d = idx - h * D;
    const float base = m_s[h] == -INFINITY ? 0.0f : m_s[h];
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w)
      O = fmaf(exp2f(red_m[w * HC + h] - base), red_acc[(w * HC + h) * RP + d], O);
    red_acc[h * RP + d] = O;  // in place: this thread alone reads and writes (h, d)
  }
  __syncthreads();
  // slots 1-3 of red_acc are free once the warps' results are merged into slot 0
  finish_cta<QT>(p, done, h0, nh, red_acc, RP, m_s, l_s, red_acc + HC * RP, 3 * HC * RP);
  if (!kPrefetch) has = sched_next<kTcTile>(p, sched);
  }
}

// ============================================================ FP8 tensor-core kernel
// head_dim = 128, e4m3 pages, bf16/f16 query. Both products run as FP8 MMAs
// (mma.m16n8k32.e4m3, fp32 accumulate), so pages are never converted:
//   * S^T = K Q^T: K's A fragments come straight out of ldmatrix; the query is split
//     into e4m3 hi + lo parts (q ~ hi + lo to ~8 significant bits) and both are applied;
//   * O^T = V^T P^T: V^T's A fragments are assembled from ldmatrix.trans words with one
//     byte permute each, using a token permutation that P^T's fragments share;
//     P is split into e4m3 hi + lo parts from f16. P is taken relative to the tile's
//     own maximum (x 256), so small probabilities keep their precision: a warp keeps
//     its accumulators relative to a per-head reference that follows the tile maxima
//     (never more than 2^24 below the running maximum) and rescales them when it moves.
// Each warp handles 32 tokens of a 128-token stage (two 16-token M tiles for S^T, one
// k32 step for PV).
__device__ __forceinline__ void mma_e4m3(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// f16x2 (x = low half) -> two e4m3 bytes (low byte from x), round to nearest even.
__device__ __forceinline__ uint32_t f16x2_to_e4m3x2(uint32_t h) {
  __half2_raw r;
  r.x = (unsigned short)(h & 0xffffu);
  r.y = (unsigned short)(h >> 16);
  return (uint32_t)__nv_cvt_halfraw2_to_fp8x2(r, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  const __half2 d = __hsub2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&d);
}

// Four floats -> e4m3 hi bytes and e4m3 bytes of the residual x - hi (byte i = x[i]).
__device__ __forceinline__ void split_e4m3x4(const float (&x)[4], uint32_t& hi, uint32_t& lo) {
  hi = lo = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint8_t h = f32_to_e4m3(x[i]);
    __nv_fp8_e4m3 hv;
    hv.__x = h;
    const uint8_t l = f32_to_e4m3(x[i] - to_f32(hv));
    hi |= (uint32_t)h << (8 * i);
    lo |= (uint32_t)l << (8 * i);
  }
}

constexpr int kF8Tile = 128;  // tokens per stage: 4 warps x 32

template <int NT>
constexpr size_t f8_epilogue_bytes() { return tc_epilogue_bytes<NT>(); }
template <int NT, int STAGES>
constexpr size_t f8_front_bytes() {
  constexpr size_t ring = (size_t)STAGES * 2 * kF8Tile * kTcD;
  return ring > f8_epilogue_bytes<NT>() ? ring : f8_epilogue_bytes<NT>();
}
template <int NT, int STAGES, bool kPT = false>
constexpr size_t f8_smem_bytes() {  // + valid flags + staged block table + query rows (+ row scales)
  return f8_front_bytes<NT, STAGES>() + (size_t)STAGES * kF8Tile + kMaxBtSmem * 4 +
         (size_t)8 * NT * kTcD * 2 + (kPT ? (size_t)STAGES * 2 * kF8Tile * 4 : 0);
}

// kPT: e4m3 pages with a scale per (page, row, kv head). S^T rows are multiplied by
// their token's K scale. P is multiplied by its token's V scale divided by 2^e, where
// 2^e bounds the tile's largest V scale, so that P stays in e4m3's range. O is kept in
// units of 2^e (rescaled by a power of two when a tile's e differs from the last one)
// and multiplied by 2^e in the merge. The softmax denominator uses the unscaled P.
template <typename QT, int NT, int STAGES, int MINB, bool kPT = false>
__global__ void __launch_bounds__(kThreads, MINB)
paged_decode_fp8mma_kernel(const DecodeParams p) {
  constexpr int D = kTcD;
  constexpr int ROWB = D;         // bytes per e4m3 token row
  constexpr int TILE_BYTES = kF8Tile * ROWB;
  constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  constexpr size_t FRONT = f8_front_bytes<NT, STAGES>();

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* valid = smem + FRONT;                                  // [STAGES][kF8Tile]
  int* bt_s = reinterpret_cast<int*>(valid + STAGES * kF8Tile);   // [kMaxBtSmem]
  QT* q_s = reinterpret_cast<QT*>(bt_s + kMaxBtSmem);              // [8 * NT][D]
  float* rs_s = reinterpret_cast<float*>(q_s + 8 * NT * D);        // kPT: [STAGES][2][kF8Tile]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  // Segment hand-over as in paged_decode_tc_kernel: the next segment's first tiles are
  // issued before this segment's epilogue, which runs in the stage of its last tile.
  constexpr bool kPrefetch = f8_epilogue_bytes<NT>() <= (size_t)STAGE_BYTES;
  const int64_t row_stride = (int64_t)p.num_kv_heads * ROWB;
  const bool one_page_per_tile = p.bs_shift >= 7;  // power-of-two block_size >= 128
  __shared__ SchedState sched;
  sched_init<kF8Tile>(p, sched);
  bool has = sched_next<kF8Tile>(p, sched);
  bool prefetched = false;
  int gt = 0;  // tiles begun by this CTA before the current segment
  BlockSlice slice{0, 0};
  while (has) {
  const TokRange rng{sched.cur.begin, sched.cur.end};
  const int seq = sched.cur.seq;
  const int kvh = sched.cur.y / p.head_groups;
  const int hgrp = sched.cur.y - kvh * p.head_groups;
  const int h0 = kvh * p.group + hgrp * p.heads_per_cta;
  const int nh = min(p.heads_per_cta, p.group - hgrp * p.heads_per_cta);
  const bool count_invalid = (kvh == 0 && hgrp == 0);

  const int ntiles = (rng.end - rng.begin + kF8Tile - 1) / kF8Tile;
  if (!prefetched) {
    slice = stage_block_table(p, seq, rng, bt_s, count_invalid);
    __syncthreads();
  }

  const int64_t head_off = (int64_t)kvh * ROWB;
  auto load_tile = [&](int it) {
    const int stage = (gt + it) % STAGES;
    uint8_t* kd = smem + stage * STAGE_BYTES;
    load_kv_tile<kF8Tile, ROWB, true>(p, seq, slice, bt_s, rng, rng.begin + it * kF8Tile, kd,
                                kd + TILE_BYTES, valid + stage * kF8Tile, row_stride, head_off,
                                one_page_per_tile, kPT ? rs_s + stage * 2 * kF8Tile : nullptr, kvh);
  };

  if (!prefetched) {
    load_q_rows<QT>(p, seq, h0, nh, q_s);
    cp_async_commit();
    // Everything above (schedule scan, block-table slice, query rows) may overlap the
    // previous kernel of a programmatic launch; the pages it may have written are read
    // only after it has completed.
    pdl_wait();
#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
      if (s < ntiles) load_tile(s);
      cp_async_commit();
    }
  }

  // ---- query as e4m3 hi + lo B fragments: b0 = d 32kq + 4tig + i, b1 = d 32kq + 16 + 4tig + i
  cp_async_wait<STAGES - 1>();  // the query rows' group (older than the tiles')
  __syncthreads();
  auto qval = [&](int row, int d) -> float { return row < nh ? to_f32(q_s[row * D + d]) : 0.0f; };
  float qmax = 0.0f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int kq = 0; kq < D / 32; ++kq)
#pragma unroll
      for (int half = 0; half < 2; ++half)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          qmax = fmaxf(qmax, fabsf(qval(nt * 8 + g, 32 * kq + 16 * half + 4 * tig + i)));
  qmax = warp_max(qmax);
  float qs = 1.0f;  // power of two: max |q| * qs in [128, 256), inside e4m3's range
  if (qmax > 0.0f && isfinite(qmax)) {
    int ex;
    frexpf(qmax, &ex);
    qs = ldexpf(1.0f, 8 - ex);
  }
  uint32_t qh[NT][D / 32][2], ql[NT][D / 32][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int kq = 0; kq < D / 32; ++kq)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = qval(nt * 8 + g, 32 * kq + 16 * half + 4 * tig + i) * qs;
        split_e4m3x4(x, qh[nt][kq][half], ql[nt][kq][half]);
      }
  const float sc = p.qk_scale_log2 * (kPT ? 1.0f : __ldg(p.k_scale)) / qs;
  int v_exp = 0;  // kPT: O is held in units of 2^v_exp

  // per-warp state for heads nt*8 + 2tig + e: running max, accumulator reference, l
  float m_run[NT][2], q_ref[NT][2], l_run[NT][2];
  float o[NT][D / 16][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt][0] = m_run[nt][1] = -INFINITY;
    q_ref[nt][0] = q_ref[nt][1] = -INFINITY;
    l_run[nt][0] = l_run[nt][1] = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 16; ++j) o[nt][j][0] = o[nt][j][1] = o[nt][j][2] = o[nt][j][3] = 0.0f;
  }

  const int lrow = lane & 7;
  const int lmat = lane >> 3;
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    if (it + STAGES - 1 < ntiles) load_tile(it + STAGES - 1);
    cp_async_commit();

    const int stage = (gt + it) % STAGES;
    const uint32_t kbase = smem_u32(smem + stage * STAGE_BYTES);
    const uint32_t vbase = kbase + TILE_BYTES;
    const uint8_t* vld = valid + stage * kF8Tile;

    // ---- S^T for the warp's two 16-token M tiles (independent chains); the hi and lo
    // query parts accumulate into the same registers
    float s[NT][2][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) s[nt][mt][i] = 0.0f;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      // matrices: (tokens 0-7, chunk 2kq) (tokens 8-15, 2kq) (0-7, 2kq+1) (8-15, 2kq+1)
      const int r = warp * 32 + mt * 16 + ((lmat & 1) << 3) + lrow;
#pragma unroll
      for (int kq = 0; kq < D / 32; ++kq) {
        const int lc = 2 * kq + (lmat >> 1);
        uint32_t a[4];
        ldmatrix_x4(kbase + r * ROWB + ((lc ^ lrow) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_e4m3(s[nt][mt], a, qh[nt][kq][0], qh[nt][kq][1]);
          mma_e4m3(s[nt][mt], a, ql[nt][kq][0], ql[nt][kq][1]);
        }
      }
    }

    // ---- softmax update and P^T (e4m3 hi + lo) B fragments
    // Per token of this thread: the score multiplier and an additive -inf for rows that
    // were not loaded, so each score costs one FFMA (0 * c - inf = -inf for those rows,
    // whose K bytes and scales are zero-filled).
    float cmul[2][2], cbias[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      cbias[mt][0] = vld[warp * 32 + mt * 16 + g] != 0 ? 0.0f : -INFINITY;
      cbias[mt][1] = vld[warp * 32 + mt * 16 + g + 8] != 0 ? 0.0f : -INFINITY;
    }
    // kPT: this thread's tokens' K scales and V scales / 2^e. O is per warp, so e comes
    // from the largest V scale of the warp's own 32 tokens (vm < 2^e). e is sticky: it
    // rises when a tile needs more range and falls only when the tile's bound is more
    // than 4 binades lower, so O is rarely rescaled, while P * vs / 2^e stays below 2^8
    // (inside e4m3's range) and within 2^-4 of it for the split's precision.
    float vsv[2][2];
    float o_rescale = 1.0f;
    if constexpr (kPT) {
      const float* rs = rs_s + stage * 2 * kF8Tile;
      float vm = 0.0f;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int tok = warp * 32 + mt * 16 + g + 8 * rr;
          cmul[mt][rr] = sc * rs[tok];
          vsv[mt][rr] = rs[kF8Tile + tok];
          vm = fmaxf(vm, vsv[mt][rr]);
        }
      // the warp's largest scale: scales are >= +0, so their bit patterns order like the
      // values and one integer reduction finds it; its exponent field gives the bound,
      // kept in [-126, 126] so that 2^-e and the power-of-two rescales are built from bits
      const uint32_t vb = __reduce_max_sync(0xffffffffu, __float_as_uint(vm));
      int e = v_exp;
      if (vb != 0u && (vb >> 23) < 0xffu) e = min((int)(vb >> 23) - 126, 126);
      if (it == 0) {
        v_exp = e;  // O is still zero
      } else if (e > v_exp || e < v_exp - 4) {
        const int d = max(min(v_exp - e, 127), -126);
        o_rescale = __uint_as_float((uint32_t)(d + 127) << 23);  // 2^(v_exp - e)
        v_exp = e;
      }
      const float inv = __uint_as_float((uint32_t)(127 - v_exp) << 23);  // 2^-v_exp
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) vsv[mt][rr] *= inv;
    } else {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) cmul[mt][0] = cmul[mt][1] = sc;
    }
    uint32_t ph[NT][2], pl[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float x[2][4];  // [mt][e + 2r], r = token g / g+8
      float f[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int rr = 0; rr < 2; ++rr)
            x[mt][e + 2 * rr] = fmaf(s[nt][mt][e + 2 * rr], cmul[mt][rr], cbias[mt][rr]);
        float mx = fmaxf(fmax3(x[0][e], x[0][e + 2], x[1][e]), x[1][e + 2]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run[nt][e], mx);
        const float q_new = mx == -INFINITY ? q_ref[nt][e] : fmaxf(mx, m_new - 24.0f);
        f[e] = q_ref[nt][e] == -INFINITY ? 1.0f : exp2f(q_ref[nt][e] - q_new);
        m_run[nt][e] = m_new;
        q_ref[nt][e] = q_new;
        // P = 2^(x - q_new + 8) <= 2^8; q_new is -inf only when every x is, and then
        // 2^(-inf) = +0
        const float qn8 = q_new == -INFINITY ? 0.0f : q_new - 8.0f;
        float lsum = 0.0f;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int i = e + 2 * rr;
            const float pv = ex2_approx(x[mt][i] - qn8);
            x[mt][i] = kPT ? pv * vsv[mt][rr] : pv;
            lsum += pv;
          }
        l_run[nt][e] = fmaf(l_run[nt][e], f[e], lsum);
        if (kPT) f[e] *= o_rescale;  // O into the units of this tile's V scales
      }
      if (f[0] != 1.0f || f[1] != 1.0f) {
        const uint64_t f2 = f2_pack(f[0], f[1]);  // accumulator pairs: (head 2tig, 2tig + 1)
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
          f2_unpack(f2_mul(f2_pack(o[nt][j][0], o[nt][j][1]), f2), o[nt][j][0], o[nt][j][1]);
          f2_unpack(f2_mul(f2_pack(o[nt][j][2], o[nt][j][3]), f2), o[nt][j][2], o[nt][j][3]);
        }
      }
      // P^T fragments: movmatrix gives (head g; tokens 2tig, 2tig+1) and (head g; tokens
      // 8+2tig, 9+2tig) of an M tile; their bytes are the k order of the V^T fragments
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint32_t x0 = movmatrix_trans(pack2<f16>(x[mt][0], x[mt][1]));
        const uint32_t x1 = movmatrix_trans(pack2<f16>(x[mt][2], x[mt][3]));
        const uint32_t h0 = f16x2_to_e4m3x2(x0), h1 = f16x2_to_e4m3x2(x1);
        const uint32_t l0 = f16x2_to_e4m3x2(hsub2_u32(x0, e4m3x2_to_f16x2((uint16_t)h0)));
        const uint32_t l1 = f16x2_to_e4m3x2(hsub2_u32(x1, e4m3x2_to_f16x2((uint16_t)h1)));
        ph[nt][mt] = h0 | (h1 << 16);
        pl[nt][mt] = l0 | (l1 << 16);
      }
    }

    // ---- O^T += V^T P^T over the warp's 32 tokens, one 16-row head_dim chunk per MMA pair.
    // ldmatrix.m16n16.x2.trans.b8 hands out the A fragments of V^T directly (lane l gets
    // rows g = l / 4 and g + 8 of the d chunk, K indices 4 tig .. 4 tig + 3 of each 16):
    // lane l < 16 addresses the row of K index l of the first 16, lane 16 + l that of K
    // index 16 + l. K index 4 tig + j is token 8 (j >> 1) + 2 tig + (j & 1), the token
    // order of the P^T fragments that movmatrix produces; O^T's rows are d = 16c + g and
    // 16c + g + 8.
    {
      const int kk = lane & 15;
      const int tok = warp * 32 + (lane & 16) + ((kk >> 1) & 1) * 8 + 2 * (kk >> 2) + (kk & 1);
      const uint32_t vrow = vbase + tok * ROWB;
      const int sw = v_swizzle_key(tok);
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        uint32_t a[4];
        ldmatrix_b8_x2_trans(vrow + ((c ^ sw) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_e4m3(o[nt][c], a, ph[nt][0], ph[nt][1]);
          mma_e4m3(o[nt][c], a, pl[nt][0], pl[nt][1]);
        }
      }
    }
  }
  gt += ntiles;

  // ---- hand over to the next segment, then merge this one
  const Seg done = sched.cur;
  uint8_t* scratch = smem;
  if (kPrefetch) {
    has = sched_next<kF8Tile>(p, sched);  // its barrier: every warp is done with the ring
    prefetched = false;
    if (has) {
      const TokRange nr{sched.cur.begin, sched.cur.end};
      const int nkvh = sched.cur.y / p.head_groups;
      const int nhg = sched.cur.y - nkvh * p.head_groups;
      const int nt2 = (nr.end - nr.begin + kF8Tile - 1) / kF8Tile;
      slice = stage_block_table(p, sched.cur.seq, nr, bt_s, nkvh == 0 && nhg == 0);
      __syncthreads();
      load_q_rows<QT>(p, sched.cur.seq, nkvh * p.group + nhg * p.heads_per_cta,
                      min(p.heads_per_cta, p.group - nhg * p.heads_per_cta), q_s);
      cp_async_commit();
#pragma unroll
      for (int s = 0; s < STAGES - 1; ++s) {
        if (s < nt2) {
          uint8_t* kd = smem + ((gt + s) % STAGES) * STAGE_BYTES;
          load_kv_tile<kF8Tile, ROWB, true>(p, sched.cur.seq, slice, bt_s, nr, nr.begin + s * kF8Tile,
                                      kd, kd + TILE_BYTES, valid + ((gt + s) % STAGES) * kF8Tile,
                                      row_stride, (int64_t)nkvh * ROWB, one_page_per_tile,
                                      kPT ? rs_s + ((gt + s) % STAGES) * 2 * kF8Tile : nullptr, nkvh);
        }
        cp_async_commit();
      }
      prefetched = true;
    }
    scratch = smem + ((gt + STAGES - 1) % STAGES) * STAGE_BYTES;  // stage of the last tile
  } else {
    cp_async_wait<0>();
    __syncthreads();
  }

  // ---- merge the 4 warps (reference q_ref plays the role of m; the x256 cancels)
  constexpr int RP = D + 4;
  constexpr int HC = 8 * NT;
  float* red_acc = reinterpret_cast<float*>(scratch);
  float* red_m = red_acc + 4 * HC * RP;
  float* red_l = red_m + 4 * HC;
  float* m_s = red_l + 4 * HC;
  float* l_s = m_s + HC;
  // kPT: each warp's O is in units of its own 2^v_exp (v_exp in [-126, 126]); it goes
  // to shared memory in absolute units
  const float o_unit = kPT ? __uint_as_float((uint32_t)(v_exp + 127) << 23) : 1.0f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = l_run[nt][e];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      const int head = nt * 8 + 2 * tig + e;
      float* ra = red_acc + (warp * HC + head) * RP;
#pragma unroll
      for (int j = 0; j < D / 16; ++j) {
        ra[16 * j + g] = kPT ? o[nt][j][e] * o_unit : o[nt][j][e];
        ra[16 * j + g + 8] = kPT ? o[nt][j][e + 2] * o_unit : o[nt][j][e + 2];
      }
      if (g == 0) {
        red_m[warp * HC + head] = q_ref[nt][e];
        red_l[warp * HC + head] = l;
      }
    }
  __syncthreads();
  if (tid < nh) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, red_m[w * HC + tid]);
    const float base = M == -INFINITY ? 0.0f : M;
    float L = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) L = fmaf(exp2f(red_m[w * HC + tid] - base), red_l[w * HC + tid], L);
    m_s[tid] = M;
    l_s[tid] = L;
  }
  __syncthreads();
  for (int idx = tid; idx < nh * D; idx += kThreads) {
    const int h = idx / D, d = idx - h * D;
    const float base = m_s[h] == -INFINITY ? 0.0f : m_s[h];
    float O = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w)
      O = fmaf(exp2f(red_m[w * HC + h] - base), red_acc[(w * HC + h) * RP + d], O);
    red_acc[h * RP + d] = O;
  }
  __syncthreads();
  // slots 1-3 of red_acc are free once the warps' results are merged into slot 0
  finish_cta<QT>(p, done, h0, nh, red_acc, RP, m_s, l_s, red_acc + HC * RP, 3 * HC * RP);
  if (!kPrefetch) has = sched_next<kF8Tile>(p, sched);
  }
}

// ============================================================ host side
struct SplitPlan {
  int num_splits;
  int chunk;
};

inline int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// Fixed split plan, shapes only (used for a forced num_splits and when the balanced
// schedule's arithmetic bound fails): the number of CTAs per (seq, kv head) is sized so
// the grid covers several waves of the 148 SMs at two resident CTAs each, with chunks of
// at most 1024 tokens and at least 128 tokens.
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

// Balanced schedule bound: at most kMaxResident CTAs (B200: 148 SMs x 4).
constexpr int kMaxResident = kNumSMs * 4;

// Items charged per unit in the balanced schedule of the tensor-core kernels, ahead of
// its tiles: a segment's fixed cost (hand-over, the 4 warps' merge, the partial write)
// is about that many tiles of streaming, so ranks that cross into more units get fewer
// tiles and all ranks finish together.
#ifndef MKV_DECODE_UNIT_COST
#define MKV_DECODE_UNIT_COST 3
#endif
constexpr int kUnitCost = MKV_DECODE_UNIT_COST;

// The balanced schedule serves num_splits = 0 unless its work-item arithmetic
// (W * G < 2^62 with W <= units * (cap / 32 + 1)) could overflow.
bool use_balanced(int num_seqs, int num_kv_heads, int head_groups, int block_size,
                  int max_blocks, int num_splits) {
  if (num_splits != 0) return false;
  const double units = (double)num_seqs * num_kv_heads * head_groups;
  const double items = units * ((double)max_blocks * block_size / 32.0 + 1.0 + kUnitCost);
  return items * kMaxResident < 4.0e18;
}

// Work items per CTA at least: few enough CTAs per unit that a unit has at most
// kMaxSplits partials (bounding the merge's work). No larger minimum: a persistent CTA
// without work exits at once, while fewer CTAs would serialise small units (256
// one-token sequences: 30.4 us with >= 256 tokens per CTA, 8 us with one tile).
int min_tiles_for(int tile, int block_size, int max_blocks) {
  const int64_t cap_tiles = ((int64_t)max_blocks * block_size + tile - 1) / tile;
  const int64_t by_merge = (cap_tiles + kMaxSplits - 3) / (kMaxSplits - 2);
  return (int)(by_merge > 1 ? by_merge : 1);
}

// Workspace layout (each part 256-byte aligned): partial accumulators, partial (m, l),
// arrival counters. Fixed splits: one partial per (sequence, head, split). Balanced:
// 2 * kMaxResident slots of heads_per_cta partials.
struct WorkspaceLayout {
  size_t acc, ml, ctr, total;
};
WorkspaceLayout workspace_layout(int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                                 int num_splits, bool balanced) {
  WorkspaceLayout w{0, 0, 0, 0};
  if (!balanced && num_splits <= 1) return w;
  const int group = num_heads / num_kv_heads;
  const int hpc = group < kMaxHeadsPerCta ? group : kMaxHeadsPerCta;
  const size_t n = balanced ? (size_t)2 * kMaxResident * hpc
                            : (size_t)num_seqs * num_heads * num_splits;
  const size_t groups = (size_t)num_seqs * num_kv_heads * head_groups_for(group);
  w.acc = 0;
  w.ml = round_up((int64_t)(n * head_dim * sizeof(float)), 256);
  w.ctr = w.ml + round_up((int64_t)(n * 2 * sizeof(float)), 256);
  w.total = w.ctr + round_up((int64_t)(groups * sizeof(unsigned int)), 256);
  return w;
}

// The kernel's dynamic shared memory opt-in, once per kernel and CUDA context.
template <auto Kernel>
int ensure_smem(size_t bytes, int device) {
  (void)device;
  return ensure_dynamic_smem((const void*)Kernel, (int)bytes,
                             "cudaFuncSetAttribute(max dynamic smem)");
}

// Resident CTAs of Kernel at `smem` bytes on `device` (occupancy x SMs), cached per device.
constexpr int kMaxDevices = 64;
template <auto Kernel>
int resident_ctas(size_t smem, int device, int* out) {
  static std::mutex mu;
  static size_t key[kMaxDevices];
  static int val[kMaxDevices];
  const bool cacheable = device >= 0 && device < kMaxDevices;
  if (cacheable) {
    std::lock_guard<std::mutex> lock(mu);
    if (val[device] > 0 && key[device] == smem) {
      *out = val[device];
      return MKV_OK;
    }
  }
  int occ = 0, sms = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, Kernel, kThreads, smem);
  if (e != cudaSuccess) return cuda_status(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return cuda_status(e, "cudaDeviceGetAttribute(SM count)");
  int g = occ * sms;
  if (g > kMaxResident) g = kMaxResident;
  if (g < 1) g = 1;
  if (cacheable) {
    std::lock_guard<std::mutex> lock(mu);
    key[device] = smem;
    val[device] = g;
  }
  *out = g;
  return MKV_OK;
}

// Grid of the launch: (splits, units per sequence, sequences) for fixed splits, or the
// resident CTAs of the kernel for the balanced schedule (which also fills p's fields).
template <auto Kernel>
int launch_decode(DecodeParams p, int tile, size_t smem, cudaStream_t stream, int device,
                  const char* what) {
  dim3 grid(p.num_splits, p.num_kv_heads * p.head_groups, p.num_seqs);
  if (p.balanced) {
    int g = 0;
    int st = resident_ctas<Kernel>(smem, device, &g);
    if (st != MKV_OK) return st;
    p.sched_ctas = g;
    p.min_tiles = min_tiles_for(tile, p.block_size, p.max_blocks);
    p.unit_cost = tile == kGenTile ? 0 : kUnitCost;
    grid = dim3(g, 1, 1);
  }
  if (p.pdl) {  // may start while the previous kernel of the stream still runs
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, Kernel, p), what);
  }
  Kernel<<<grid, kThreads, smem, stream>>>(p);
  return cuda_status(cudaGetLastError(), what);
}

template <typename QT, typename CT>
int launch_generic(const DecodeParams& p, cudaStream_t stream, int device) {
  const size_t smem = generic_smem_bytes(p.head_dim, sizeof(CT));
  // opt in once to the largest size this instantiation can use (head_dim 256)
  int st = ensure_smem<paged_decode_generic_kernel<QT, CT>>(generic_smem_bytes(256, sizeof(CT)),
                                                            device);
  if (st != MKV_OK) return st;
  return launch_decode<paged_decode_generic_kernel<QT, CT>>(p, kGenTile, smem, stream, device,
                                                            "paged_decode_generic launch");
}

// Pipeline depth and CTAs per SM: 16-bit pages 2 stages x 32 KB (3 CTAs/SM), e4m3
// pages 3 stages x 16 KB (4 CTAs/SM).
// Measured on B200 (config 3, bf16): 2 stages x 3 CTAs/SM 6.05 TB/s, 3 x 2 5.29 TB/s,
// 4 x 1 2.99 TB/s -- the decode is bound by resident warps, not by ring depth.
#ifndef MKV_TC16_STAGES
#define MKV_TC16_STAGES 2
#define MKV_TC16_MINB 3
#endif
#ifndef MKV_TC8_STAGES
#define MKV_TC8_STAGES 3
#define MKV_TC8_MINB 4
#endif
template <typename CT> struct TcConfig;
template <> struct TcConfig<bf16> { static constexpr int kStages = MKV_TC16_STAGES, kMinBlocks = MKV_TC16_MINB; };
template <> struct TcConfig<f16> { static constexpr int kStages = MKV_TC16_STAGES, kMinBlocks = MKV_TC16_MINB; };
template <> struct TcConfig<int8_t> { static constexpr int kStages = MKV_TC8_STAGES, kMinBlocks = MKV_TC8_MINB; };

template <typename QT, typename CT, int NT, bool kPT>
int launch_tc_nt(const DecodeParams& p, cudaStream_t stream, int device) {
  constexpr int S = TcConfig<CT>::kStages, MB = TcConfig<CT>::kMinBlocks;
  constexpr size_t smem = tc_smem_bytes<CT, NT, S>();
  int st = ensure_smem<paged_decode_tc_kernel<QT, CT, NT, S, MB, kPT>>(smem, device);
  if (st != MKV_OK) return st;
  return launch_decode<paged_decode_tc_kernel<QT, CT, NT, S, MB, kPT>>(
      p, kTcTile, smem, stream, device, "paged_decode_tc launch");
}

// e4m3 pages with FP8 MMAs: 2 stages x 32 KB (128-token tiles), 3 CTAs/SM.
#ifndef MKV_F8_STAGES
#define MKV_F8_STAGES 2
#define MKV_F8_MINB 3
#endif
template <typename QT, int NT, bool kPT>
int launch_fp8mma_nt(const DecodeParams& p, cudaStream_t stream, int device) {
  constexpr int S = MKV_F8_STAGES, MB = MKV_F8_MINB;
  constexpr size_t smem = f8_smem_bytes<NT, S, kPT>();
  int st = ensure_smem<paged_decode_fp8mma_kernel<QT, NT, S, MB, kPT>>(smem, device);
  if (st != MKV_OK) return st;
  return launch_decode<paged_decode_fp8mma_kernel<QT, NT, S, MB, kPT>>(
      p, kF8Tile, smem, stream, device, "paged_decode_fp8mma launch");
}
template <typename QT, bool kPT = false>
int launch_fp8mma(const DecodeParams& p, cudaStream_t stream, int device) {
  return p.heads_per_cta > 8 ? launch_fp8mma_nt<QT, 2, kPT>(p, stream, device)
                             : launch_fp8mma_nt<QT, 1, kPT>(p, stream, device);
}

template <typename QT, typename CT, bool kPT = false>
int launch_tc(const DecodeParams& p, cudaStream_t stream, int device) {
  return p.heads_per_cta > 8 ? launch_tc_nt<QT, CT, 2, kPT>(p, stream, device)
                             : launch_tc_nt<QT, CT, 1, kPT>(p, stream, device);
}

int decode_impl(const char* fn, const void* query, int64_t q_sb, int64_t q_sh, int q_dtype,
                const void* k_cache, const void* v_cache, int cache_dtype, const float* k_scale,
                const float* v_scale, const float* k_scales, const float* v_scales,
                int64_t num_blocks, int block_size, const void* bt,
                int bt_type, int64_t bt_sb, int max_blocks, const void* ctx, int ctx_type,
                int num_seqs, int num_heads, int num_kv_heads, int head_dim, float scale,
                void* out, int64_t o_sb, int64_t o_sh, void* workspace, size_t ws_bytes,
                uint32_t* counters, size_t counters_bytes, int num_splits, unsigned flags,
                int32_t* invalid, void* stream) {
  clear_error();
  if (flags & ~(unsigned)MKV_DECODE_OVERLAP_PREVIOUS)
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: unknown flags 0x%x", fn, flags);
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
  if ((int64_t)max_blocks * block_size >= ((int64_t)1 << 31) || num_blocks >= ((int64_t)1 << 31))
    return set_error(MKV_ERR_UNSUPPORTED,
                     "%s: max_num_blocks * block_size and num_blocks must be < 2^31", fn);
  if (head_dim % 16 != 0 || head_dim > 256)
    return set_error(MKV_ERR_UNSUPPORTED,
                     "%s: head_dim must be a multiple of 16 and at most 256 (got %d)", fn,
                     head_dim);
  const bool fp8_cache = cache_dtype == MKV_DTYPE_FP8_E4M3;
  const bool per_token = k_scales != nullptr || v_scales != nullptr;
  if (per_token && (!k_scales || !v_scales))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: both k_scales and v_scales are needed", fn);
  if (per_token && (((uintptr_t)k_scales & 3u) || ((uintptr_t)v_scales & 3u)))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: scales must be 4-byte aligned", fn);
  if (per_token && !fp8_cache && cache_dtype != MKV_DTYPE_INT8)
    return set_error(MKV_ERR_UNSUPPORTED,
                     "%s: per-token scales need an FP8_E4M3 or INT8 cache (got %d)", fn,
                     cache_dtype);
  if (fp8_cache && !per_token && (!k_scale || !v_scale))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: FP8 cache needs k_scale and v_scale", fn);
  if (cache_dtype == MKV_DTYPE_INT8 && !per_token)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: an INT8 cache needs per-token scales", fn);
  if (!fp8_cache && !per_token && cache_dtype != q_dtype)
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
  const bool balanced =
      use_balanced(num_seqs, num_kv_heads, hgs, block_size, max_blocks, num_splits);
  const SplitPlan sp = plan_splits(num_seqs, num_kv_heads, hgs, block_size, max_blocks, num_splits);
  const WorkspaceLayout wl =
      workspace_layout(num_seqs, num_heads, num_kv_heads, head_dim, sp.num_splits, balanced);
  // With a caller-kept counter buffer the workspace holds the partials only.
  const size_t counter_need = wl.total ? wl.total - wl.ctr : 0;
  const bool own_counters = counters != nullptr && counter_need > 0;
  const size_t ws_need = own_counters ? wl.ctr : wl.total;
  if (ws_need > 0 && (workspace == nullptr || ws_bytes < ws_need))
    return set_error(MKV_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", fn,
                     ws_need, workspace ? ws_bytes : (size_t)0);
  if (ws_need > 0 && ((uintptr_t)workspace & 15u))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: workspace must be 16-byte aligned", fn);
  if (own_counters && (counters_bytes < counter_need || ((uintptr_t)counters & 3u)))
    return set_error(MKV_ERR_WORKSPACE, "%s: counter buffer of %zu bytes (4-byte aligned) needed, %zu given",
                     fn, counter_need, counters_bytes);

  DecodeParams p;
  p.q = query;
  p.q_sb = q_sb;
  p.q_sh = q_sh;
  {
    const int64_t qeb = q_dtype == MKV_DTYPE_F32 ? 4 : 2;
    p.q_vec16 = ((uintptr_t)query % 16 == 0) && (q_sb * qeb) % 16 == 0 && (q_sh * qeb) % 16 == 0;
  }
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
  p.k_scale = fp8_cache && !per_token ? k_scale : nullptr;
  p.v_scale = fp8_cache && !per_token ? v_scale : nullptr;
  p.k_scales = per_token ? k_scales : nullptr;
  p.v_scales = per_token ? v_scales : nullptr;
  p.out = out;
  p.o_sb = o_sb;
  p.o_sh = o_sh;
  p.num_splits = sp.num_splits;
  p.chunk = sp.chunk;
  p.balanced = balanced ? 1 : 0;
  p.sched_ctas = 0;  // set at launch from the kernel's occupancy
  p.min_tiles = 1;
  p.unit_cost = 0;
  uint8_t* ws = (uint8_t*)workspace;
  p.part_acc = wl.total ? (float*)(ws + wl.acc) : nullptr;
  p.part_ml = wl.total ? (float*)(ws + wl.ml) : nullptr;
  p.arrivals = wl.total ? (own_counters ? (unsigned int*)counters : (unsigned int*)(ws + wl.ctr))
                        : nullptr;
  p.invalid = invalid;
  p.pdl = (flags & MKV_DECODE_OVERLAP_PREVIOUS) ? 1 : 0;

  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  cudaStream_t s = (cudaStream_t)stream;
  // Arrival counters start at zero. The kernel leaves them at zero, so a caller-kept
  // counter buffer (zeroed once, used for nothing else) needs no clear.
  if (wl.total && !own_counters) {
    e = cudaMemsetAsync(ws + wl.ctr, 0, wl.total - wl.ctr, s);
    if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync(arrival counters)");
  }

  const bool tc_ok = head_dim == kTcD && q_dtype != MKV_DTYPE_F32;
  if (per_token) {  // 8-bit pages with per-(page, row, kv head) scales
    const bool i8 = cache_dtype == MKV_DTYPE_INT8;
    // e4m3: FP8 MMAs with the scales applied to S and P; int8: pages converted to f16
    if (tc_ok && q_dtype == MKV_DTYPE_BF16)
      return i8 ? launch_tc<bf16, int8_t, true>(p, s, device) : launch_fp8mma<bf16, true>(p, s, device);
    if (tc_ok && q_dtype == MKV_DTYPE_F16)
      return i8 ? launch_tc<f16, int8_t, true>(p, s, device) : launch_fp8mma<f16, true>(p, s, device);
    switch (q_dtype) {
      case MKV_DTYPE_F32:
        return i8 ? launch_generic<float, int8_t>(p, s, device) : launch_generic<float, fp8>(p, s, device);
      case MKV_DTYPE_F16:
        return i8 ? launch_generic<f16, int8_t>(p, s, device) : launch_generic<f16, fp8>(p, s, device);
      default:
        return i8 ? launch_generic<bf16, int8_t>(p, s, device) : launch_generic<bf16, fp8>(p, s, device);
    }
  }
  if (tc_ok && !fp8_cache && q_dtype == MKV_DTYPE_BF16) return launch_tc<bf16, bf16>(p, s, device);
  if (tc_ok && !fp8_cache && q_dtype == MKV_DTYPE_F16) return launch_tc<f16, f16>(p, s, device);
  if (tc_ok && fp8_cache && q_dtype == MKV_DTYPE_BF16) return launch_fp8mma<bf16>(p, s, device);
  if (tc_ok && fp8_cache && q_dtype == MKV_DTYPE_F16) return launch_fp8mma<f16>(p, s, device);
  if (fp8_cache) {
    switch (q_dtype) {
      case MKV_DTYPE_F32: return launch_generic<float, fp8>(p, s, device);
      case MKV_DTYPE_F16: return launch_generic<f16, fp8>(p, s, device);
      default: return launch_generic<bf16, fp8>(p, s, device);
    }
  }
  switch (q_dtype) {
    case MKV_DTYPE_F32: return launch_generic<float, float>(p, s, device);
    case MKV_DTYPE_F16: return launch_generic<f16, f16>(p, s, device);
    default: return launch_generic<bf16, bf16>(p, s, device);
  }
}

// ---------------------------------------------------------------- allocation-free entry
// Built-in decode scratch for callers that cannot allocate device memory. Every device
// that loads this library holds these MKV_NOALLOC_SCRATCH_BYTES until the process ends.
// Host code only sees a shadow of this symbol: its device address is looked up with
// cudaGetSymbolAddress and passed to the kernels like any caller workspace.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MKV_NOALLOC_SCRATCH_BYTES];

// The address belongs to the CUDA context that was current when it was looked up (the
// module is loaded per context). It is cached per context, keyed on the context's
// unique ID (current_context_id): a caller's own driver-API context, or the primary
// context created again after cudaDeviceReset, gets a lookup of its own instead of an
// address from another or a destroyed context.
struct NoallocEntry {
  unsigned long long ctx_id;
  void* ptr;
};
constexpr int kNoallocCacheEntries = 64;
std::mutex g_noalloc_mu;
NoallocEntry g_noalloc_cache[kNoallocCacheEntries] = {};
int g_noalloc_next = 0;  // round-robin replacement once the cache is full

// Device address of g_noalloc_scratch in the current context, looked up on the first
// call in that context.
int noalloc_scratch(void** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  unsigned long long id = 0;
  int st = current_context_id(&id);
  if (st != MKV_OK) return st;
  if (id != 0) {
    for (const NoallocEntry& en : g_noalloc_cache)
      if (en.ptr != nullptr && en.ctx_id == id) {
        *out = en.ptr;
        return MKV_OK;
      }
  }
  // First call in this context (or no context current yet: the runtime's lookup below
  // makes the device's primary context current, and its ID is read afterwards).
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(built-in decode scratch)");
  if (id == 0) {
    st = current_context_id(&id);
    if (st != MKV_OK) return st;
    if (id == 0) return set_error(MKV_ERR_CUDA, "mkv_paged_decode_noalloc: no current CUDA context");
  }
  g_noalloc_cache[g_noalloc_next] = NoallocEntry{id, ptr};
  g_noalloc_next = (g_noalloc_next + 1) % kNoallocCacheEntries;
  *out = ptr;
  return MKV_OK;
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
  if (use_balanced(num_seqs, num_kv_heads, hgs, block_size, max_num_blocks, 0)) return 0;
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
  const bool balanced =
      use_balanced(num_seqs, num_kv_heads, hgs, block_size, max_num_blocks, num_splits);
  return workspace_layout(num_seqs, num_heads, num_kv_heads, head_dim, sp.num_splits, balanced)
      .total;
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
                     v_cache, cache_dtype, nullptr, nullptr, nullptr, nullptr, num_blocks,
                     block_size, block_tables, block_table_index_type, block_table_stride_seq, max_num_blocks, context_lens,
                     context_lens_index_type, num_seqs, num_heads, num_kv_heads, head_dim, scale,
                     out, out_stride_seq, out_stride_head, workspace, workspace_bytes, nullptr, 0,
                     num_splits, 0u, invalid_count, stream);
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
                     v_cache, MKV_DTYPE_FP8_E4M3, k_scale, v_scale, nullptr, nullptr, num_blocks, block_size,
                     block_tables, block_table_index_type, block_table_stride_seq, max_num_blocks,
                     context_lens, context_lens_index_type, num_seqs, num_heads, num_kv_heads,
                     head_dim, scale, out, out_stride_seq, out_stride_head, workspace,
                     workspace_bytes, nullptr, 0, num_splits, 0u, invalid_count, stream);
}

extern "C" int mkv_paged_decode_noalloc(const void* query, int64_t q_stride_seq,
                                        int64_t q_stride_head, int32_t q_dtype,
                                        const void* k_cache, const void* v_cache,
                                        int32_t cache_dtype, int64_t num_blocks,
                                        int32_t block_size, const void* block_tables,
                                        int32_t block_table_index_type,
                                        int64_t block_table_stride_seq, int32_t max_num_blocks,
                                        const void* context_lens, int32_t context_lens_index_type,
                                        int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                        int32_t head_dim, float scale, void* out,
                                        int64_t out_stride_seq, int64_t out_stride_head,
                                        int32_t num_splits, int32_t* invalid_count,
                                        void* stream) {
  clear_error();
  if (cache_dtype == MKV_DTYPE_FP8_E4M3)
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "mkv_paged_decode_noalloc: FP8 caches go through mkv_paged_decode_fp8");
  const size_t need = mkv_paged_decode_workspace_bytes(num_seqs, num_heads, num_kv_heads, head_dim,
                                                       block_size, max_num_blocks, num_splits);
  if (need > (size_t)MKV_NOALLOC_SCRATCH_BYTES)
    return set_error(MKV_ERR_WORKSPACE,
                     "mkv_paged_decode_noalloc: this shape needs %zu bytes of split scratch but the "
                     "built-in scratch holds %zu; pass a smaller num_splits (1 needs none) or call "
                     "mkv_paged_decode with a workspace",
                     need, (size_t)MKV_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (need > 0) {
    int st = noalloc_scratch(&scratch);
    if (st != MKV_OK) return st;
  }
  return decode_impl("mkv_paged_decode_noalloc", query, q_stride_seq, q_stride_head, q_dtype,
                     k_cache, v_cache, cache_dtype, nullptr, nullptr, nullptr, nullptr, num_blocks,
                     block_size,
                     block_tables, block_table_index_type, block_table_stride_seq, max_num_blocks,
                     context_lens, context_lens_index_type, num_seqs, num_heads, num_kv_heads,
                     head_dim, scale, out, out_stride_seq, out_stride_head, scratch,
                     scratch ? (size_t)MKV_NOALLOC_SCRATCH_BYTES : 0, nullptr, 0, num_splits, 0u,
                     invalid_count, stream);
}

extern "C" int mkv_paged_decode_quant_per_token_head(
    const void* query, int64_t q_stride_seq, int64_t q_stride_head, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t cache_dtype, const float* k_scales,
    const float* v_scales, int64_t num_blocks, int32_t block_size, const void* block_tables,
    int32_t block_table_index_type, int64_t block_table_stride_seq, int32_t max_num_blocks,
    const void* context_lens, int32_t context_lens_index_type, int32_t num_seqs,
    int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float scale, void* out,
    int64_t out_stride_seq, int64_t out_stride_head, void* workspace, size_t workspace_bytes,
    int32_t num_splits, int32_t* invalid_count, void* stream) {
  clear_error();
  const char* fn = "mkv_paged_decode_quant_per_token_head";
  if (cache_dtype != MKV_DTYPE_FP8_E4M3 && cache_dtype != MKV_DTYPE_INT8)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: cache_dtype must be FP8_E4M3 or INT8 (got %d)", fn,
                     cache_dtype);
  if (num_seqs > 0 && (!k_scales || !v_scales))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: null scale pointer", fn);
  return decode_impl(fn, query, q_stride_seq, q_stride_head, q_dtype, k_cache, v_cache,
                     cache_dtype, nullptr, nullptr, k_scales, v_scales, num_blocks, block_size,
                     block_tables, block_table_index_type, block_table_stride_seq, max_num_blocks,
                     context_lens, context_lens_index_type, num_seqs, num_heads, num_kv_heads,
                     head_dim, scale, out, out_stride_seq, out_stride_head, workspace,
                     workspace_bytes, nullptr, 0, num_splits, 0u, invalid_count, stream);
}

extern "C" int mkv_paged_decode_ex(
    const void* query, int64_t q_stride_seq, int64_t q_stride_head, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t cache_dtype, const float* k_scale,
    const float* v_scale, const float* k_scales, const float* v_scales, int64_t num_blocks,
    int32_t block_size, const void* block_tables, int32_t block_table_index_type,
    int64_t block_table_stride_seq, int32_t max_num_blocks, const void* context_lens,
    int32_t context_lens_index_type, int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
    int32_t head_dim, float scale, void* out, int64_t out_stride_seq, int64_t out_stride_head,
    void* workspace, size_t workspace_bytes, uint32_t* counters, size_t counters_bytes,
    int32_t num_splits, uint32_t flags, int32_t* invalid_count, void* stream) {
  const char* fn = "mkv_paged_decode_ex";
  clear_error();
  const bool per_token = k_scales != nullptr || v_scales != nullptr;
  if (per_token && (k_scale != nullptr || v_scale != nullptr))
    return set_error(MKV_ERR_INVALID_ARGUMENT,
                     "%s: give either per-tensor scales or per-(token, head) scales", fn);
  if (per_token && cache_dtype != MKV_DTYPE_FP8_E4M3 && cache_dtype != MKV_DTYPE_INT8)
    return set_error(MKV_ERR_UNSUPPORTED, "%s: per-token scales need an FP8_E4M3 or INT8 cache", fn);
  if (!per_token && cache_dtype != MKV_DTYPE_FP8_E4M3 && (k_scale != nullptr || v_scale != nullptr))
    return set_error(MKV_ERR_INVALID_ARGUMENT, "%s: scales given for an unquantised cache", fn);
  return decode_impl(fn, query, q_stride_seq, q_stride_head, q_dtype, k_cache, v_cache,
                     cache_dtype, per_token ? nullptr : k_scale, per_token ? nullptr : v_scale,
                     k_scales, v_scales, num_blocks, block_size, block_tables,
                     block_table_index_type, block_table_stride_seq, max_num_blocks, context_lens,
                     context_lens_index_type, num_seqs, num_heads, num_kv_heads, head_dim, scale,
                     out, out_stride_seq, out_stride_head, workspace, workspace_bytes, counters,
                     counters_bytes, num_splits, flags, invalid_count, stream);
}

extern "C" size_t mkv_paged_decode_counter_bytes(int32_t num_seqs, int32_t num_heads,
                                                 int32_t num_kv_heads, int32_t head_dim,
                                                 int32_t block_size, int32_t max_num_blocks,
                                                 int32_t num_splits) {
  if (num_seqs <= 0 || num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads != 0 ||
      head_dim <= 0 || num_splits < 0)
    return 0;
  const int hgs = head_groups_for(num_heads / num_kv_heads);
  const SplitPlan sp =
      plan_splits(num_seqs, num_kv_heads, hgs, block_size, max_num_blocks, num_splits);
  const bool balanced =
      use_balanced(num_seqs, num_kv_heads, hgs, block_size, max_num_blocks, num_splits);
  const WorkspaceLayout wl =
      workspace_layout(num_seqs, num_heads, num_kv_heads, head_dim, sp.num_splits, balanced);
  return wl.total ? wl.total - wl.ctr : 0;
}
