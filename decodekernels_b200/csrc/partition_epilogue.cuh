// Cross-warp merge at the end of a partition, shared by both partition
// kernels.  Each of W warps left, per query head h of the group, an online-
// softmax state in shared memory: the running max m (log2-scaled logits), the
// exp-sum l and the unnormalised output O = sum_t exp2(s_t - m) v_t.  The
// partition result is
//   M = max_w m_w,  den = sum_w l_w 2^(m_w - M),  o = sum_w O_w 2^(m_w - M) / den
// and is written either to `out` (single pass) or, as DecodeKernels' split-K
// kernel does (csrc/paged_attention.cuh:205-224), to the workspace row
// (seq * Hq + q_head) * P + part as (o, max logit M * ln2, den).
#pragma once

#include "decode_params.cuh"
#include "dk_ptx.cuh"

namespace dkb {

// Row stride (floats) of the per-warp output scratch: D + 4 keeps the
// fragment-ordered stores free of bank conflicts.
template <int D>
struct RedLayout {
  static constexpr int kRow = D + 4;
  static constexpr int floats(int warps) { return warps * kMaxGroup * kRow + 2 * warps * kMaxGroup; }
};

// A sequence whose whole length fits in partition 0 needs no merge: its
// result also goes straight to `out` (the merge kernel skips it), while the
// workspace row is still written so the workspace keeps the same contents.
template <typename T, int D, int WARPS>
__device__ __forceinline__ void write_partition_result(const DecodeParams& p, const float* red_o, const float* red_m,
                                                       const float* red_l, int seq, int kv_head, int part, int seq_len,
                                                       int tid, int nthreads) {
  const int group = p.group;
  const bool to_out = !p.split || (part == 0 && seq_len <= p.partition_size);
  constexpr int R = RedLayout<D>::kRow;
  for (int idx = tid; idx < group * D; idx += nthreads) {
    const int h = idx / D;
    const int d = idx - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, red_m[w * kMaxGroup + h]);
    float num = 0.0f, den = 0.0f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float e = fast_exp2(red_m[w * kMaxGroup + h] - M);  // 0 for warps that saw no token
      den = fmaf(e, red_l[w * kMaxGroup + h], den);
      num = fmaf(e, red_o[(w * kMaxGroup + h) * R + d], num);
    }
    const float o = num / den;
    const int q_head = kv_head * group + h;
    if (p.split) {
      const int64_t row = (static_cast<int64_t>(seq) * p.num_q_heads + q_head) * p.ws_partitions + part;
      p.tmp_out[row * D + d] = o;
      if (d == 0) {
        p.max_logits[row] = M * kLn2;
        p.exp_sums[row] = den;
      }
    }
    if (to_out) static_cast<T*>(p.out)[seq * p.out_stride_seq + q_head * p.out_stride_head + d] = Conv<T>::from_f32(o);
  }
}

// Zeros for the group's query heads of an empty sequence (single-pass path),
// matching csrc/paged_attention.cuh:91-105.
template <typename T, int D>
__device__ __forceinline__ void write_zero_output(const DecodeParams& p, int seq, int kv_head, int tid, int nthreads) {
  for (int idx = tid; idx < p.group * D; idx += nthreads) {
    const int h = idx / D;
    const int d = idx - h * D;
    const int q_head = kv_head * p.group + h;
    static_cast<T*>(p.out)[seq * p.out_stride_seq + q_head * p.out_stride_head + d] = Conv<T>::from_f32(0.0f);
  }
}

}  // namespace dkb
