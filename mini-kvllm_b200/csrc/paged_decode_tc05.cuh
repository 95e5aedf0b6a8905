// Persistent tcgen05 + TMA paged decode (paged_decode_tc05.cu): launch interface used by
// the decode entry points in paged_decode.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mkv {
namespace tc05 {

struct Params {
  const void* q;
  int64_t q_sb, q_sh;
  int64_t num_blocks;
  int block_size, bs_shift;
  const void* bt;
  int64_t bt_sb;
  int max_blocks, bt_i64;
  const void* ctx;
  int ctx_i64;
  int num_seqs, num_heads, num_kv_heads;
  int group, heads_per_cta, head_groups;
  float qk_scale_log2;
  const float* k_scale;
  const float* v_scale;
  void* out;
  int64_t o_sb, o_sh;
  float* part_acc;
  float* part_ml;
  unsigned int* arrivals;
  int num_splits, chunk;
  int64_t num_units;
  int32_t* invalid;
};

// True when the tcgen05 kernel handles this shape: head_dim 128, bf16/f16 query with a
// cache of the same type or e4m3, block_size a power of two >= 8, TMA encode available.
bool supported(int q_dtype, int cache_dtype, int head_dim, int block_size, int heads_per_cta);

// Encodes the K/V tensor maps and launches one CTA per SM over all work units.
int launch(const Params& p, int q_dtype, int cache_dtype, const void* k_cache,
           const void* v_cache, cudaStream_t stream, int device);

}  // namespace tc05
}  // namespace mkv
