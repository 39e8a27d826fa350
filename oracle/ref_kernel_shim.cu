// Side-by-side checker: the reference's OWN paged-attention kernels, compiled
// from its source tree in place (this file includes
// csrc/paged_attention.cuh from the DecodeKernels tree given with -I; nothing
// is copied) for sm_100a, behind a small C entry point so GPU tests can run
// them on the same inputs as this library.  TEST INFRASTRUCTURE, NOT PRODUCT.
//
// Built by oracle/build.py into oracle/_ref/libdk_ref_kernel.so only when the
// reference tree exists (the build container); the .so then travels to the
// GPU box with the rest of the tree.
#include <cstdint>

#include "paged_attention.cuh"

extern "C" {

typedef struct DkRefArgs {
  void* out;
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const int32_t* block_tables;
  const int32_t* seq_lens;
  float* tmp_out;
  float* max_logits;
  float* exp_sums;
  int64_t q_stride_seq, q_stride_head;
  int64_t out_stride_seq, out_stride_head;
  int64_t k_stride_block, k_stride_token, k_stride_head;
  int64_t v_stride_block, v_stride_token, v_stride_head;
  int64_t bt_stride;
  int32_t num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max_partitions, max_seq_len, dtype;
  float scale;
} DkRefArgs;

__attribute__((visibility("default"))) int dk_ref_paged_attention_decode(const DkRefArgs* a, void* stream) {
  dk::PagedAttnParams p{};
  p.out = a->out;
  p.q = a->q;
  p.k_cache = a->k_cache;
  p.v_cache = a->v_cache;
  p.block_tables = a->block_tables;
  p.seq_lens = a->seq_lens;
  p.tmp_out = a->tmp_out;
  p.max_logits = a->max_logits;
  p.exp_sums = a->exp_sums;
  p.q_stride_seq = a->q_stride_seq;
  p.q_stride_head = a->q_stride_head;
  p.out_stride_seq = a->out_stride_seq;
  p.out_stride_head = a->out_stride_head;
  p.k_stride_block = a->k_stride_block;
  p.k_stride_token = a->k_stride_token;
  p.k_stride_head = a->k_stride_head;
  p.v_stride_block = a->v_stride_block;
  p.v_stride_token = a->v_stride_token;
  p.v_stride_head = a->v_stride_head;
  p.bt_stride = a->bt_stride;
  p.num_seqs = a->num_seqs;
  p.num_q_heads = a->num_q_heads;
  p.num_kv_heads = a->num_kv_heads;
  p.block_size = a->block_size;
  p.max_partitions = a->max_partitions;
  p.scale = a->scale;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->dtype == 1) return dk::launch_paged_attention_decode<__nv_bfloat16>(p, a->head_dim, a->max_seq_len, s);
  return dk::launch_paged_attention_decode<__half>(p, a->head_dim, a->max_seq_len, s);
}

}  // extern "C"
