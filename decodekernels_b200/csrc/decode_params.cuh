// Parameters shared by the partition kernels and the merge kernel.
#pragma once

#include <stdint.h>

namespace dkb {

constexpr int kTileTokens = 64;      // partition-size granularity; every pipeline tile divides it
constexpr int kSubTokens = 16;       // tokens per consumer warp per tile (mma M)
constexpr int kSimtThreads = 128;
constexpr int kMergeThreads = 256;
constexpr int kMaxGroup = 8;         // query heads per KV head (mma N)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Everything a launch needs besides the TMA descriptors.  Strides are in
// elements.  Field meanings follow DecodeKernels' PagedAttnParams
// (csrc/paged_attention.cuh:39-58) plus the planner's outputs.
struct DecodeParams {
  void* out;
  const void* q;
  const void* k_cache;  // read directly by the CUDA-core path only
  const void* v_cache;
  const int* block_tables;
  const int* seq_lens;
  float* tmp_out;
  float* max_logits;
  float* exp_sums;
  int* merge_counters;  // non-null: the last partition of each (seq, kv_head) merges (no merge kernel)
  int64_t q_stride_seq, q_stride_head;
  int64_t out_stride_seq, out_stride_head;
  int64_t k_stride_block, k_stride_token, k_stride_head;
  int64_t v_stride_block, v_stride_token, v_stride_head;
  int64_t bt_stride;
  int num_seqs;
  int num_q_heads;
  int num_kv_heads;
  int group;           // num_q_heads / num_kv_heads
  int max_seq_len;     // host-side bound on seq_lens; longer lengths count as this
  int block_size;
  int num_blocks;      // cache blocks; ids outside [0, num_blocks) read as zeros
  int bs_log2;         // log2(block_size) (TMA path: power-of-two block sizes)
  int rows_log2;       // log2 of token rows per TMA box: min(block_size, tile)
  int partition_size;  // tokens per partition, a multiple of kTileTokens
  int num_partitions;  // partitions in the grid
  int ws_partitions;   // workspace row stride (capacity)
  int split;           // 1: partitions write the workspace and the merge kernel writes out
  int kv_fused;        // 1: one tensor map covers K and V (vLLM's interleaved K|V rows)
  int lse_mode;        // 1: `out` is fp32 rows [o (head_dim) | lse | 3 pad] per (seq, q_head), not T
  float scale_log2;    // softmax scale * log2(e) (* k_scale for e4m3 caches)
  float v_scale;       // e4m3 caches: V = code * v_scale (1 otherwise), applied to the partition results
  int kv_fp8;          // 1: the caches hold e4m3 bytes
};

// (partition, kv_head, seq) of this CTA in the 1-D grid, sequence-major:
// a (seq, kv_head)'s partitions are consecutive, so a long sequence's work is
// spread over the whole grid.  (Partition-major order, which pushes the
// early-exit CTAs past short sequences' ends to the back, measured 10% slower
// on skewed lengths -- it also pushes long sequences' last partitions into
// the tail -- and within 2% elsewhere.)
__device__ __forceinline__ void cta_coords(int num_partitions, int num_kv_heads, int& part, int& kv_head, int& seq) {
  const unsigned b = blockIdx.x;
  const unsigned np = static_cast<unsigned>(num_partitions);
  const unsigned pair = b / np;
  part = static_cast<int>(b - pair * np);
  seq = static_cast<int>(pair / static_cast<unsigned>(num_kv_heads));
  kv_head = static_cast<int>(pair - static_cast<unsigned>(seq) * static_cast<unsigned>(num_kv_heads));
}

}  // namespace dkb
