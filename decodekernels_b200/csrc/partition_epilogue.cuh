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

// Shared-memory scratch of the merge: per-warp output rows (row stride D + 4
// keeps the fragment-ordered stores free of bank conflicts and the rows
// 16-byte aligned), per-warp (m, l), then the per-(warp, head) merge factors
// 2^(m_w - M) / den and the per-head (M, den).
template <int D>
struct RedLayout {
  static constexpr int kRow = D + 4;
  static constexpr int floats(int warps) { return warps * kMaxGroup * kRow + 3 * warps * kMaxGroup + 2 * kMaxGroup; }
  static __device__ __forceinline__ float* o(float* red) { return red; }
  static __device__ __forceinline__ float* m(float* red, int warps) { return red + warps * kMaxGroup * kRow; }
  static __device__ __forceinline__ float* l(float* red, int warps) { return m(red, warps) + warps * kMaxGroup; }
  static __device__ __forceinline__ float* fac(float* red, int warps) { return l(red, warps) + warps * kMaxGroup; }
  static __device__ __forceinline__ float* head(float* red, int warps) { return fac(red, warps) + warps * kMaxGroup; }
};

// Merge the WARPS per-warp states already in `red` and write the result of
// this (sequence, kv_head) partition: to workspace row
// (seq * Hq + q_head) * ws_partitions + row when `to_ws`, and to `out` when
// `to_out`.  The per-head factors are computed once (by `group` threads),
// then every thread produces 4 consecutive outputs.  `sync` is the barrier of
// the `nthreads` participating threads.
template <typename T, int D, int WARPS, typename Sync>
__device__ __forceinline__ void write_merged_result(const DecodeParams& p, float* red, int seq, int kv_head, int row,
                                                    bool to_ws, bool to_out, int tid, int nthreads, Sync sync) {
  using L = RedLayout<D>;
  constexpr int R = L::kRow;
  const int group = p.group;
  const float* red_o = L::o(red);
  const float* red_m = L::m(red, WARPS);
  const float* red_l = L::l(red, WARPS);
  float* fac = L::fac(red, WARPS);
  float* head = L::head(red, WARPS);
  if (tid < group) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, red_m[w * kMaxGroup + tid]);
    float e[WARPS];
    float den = 0.0f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      e[w] = fast_exp2(red_m[w * kMaxGroup + tid] - M);  // 0 for warps that saw no token
      den = fmaf(e[w], red_l[w * kMaxGroup + tid], den);
    }
    const float inv = 1.0f / den;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) fac[w * kMaxGroup + tid] = e[w] * inv;
    head[tid] = M;
    head[kMaxGroup + tid] = den;
  }
  sync();
  constexpr int Q = D / 4;
  for (int idx = tid; idx < group * Q; idx += nthreads) {
    const int h = idx / Q;
    const int d = (idx - h * Q) * 4;
    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float f = fac[w * kMaxGroup + h];
      const float4 x = *reinterpret_cast<const float4*>(red_o + (w * kMaxGroup + h) * R + d);
      o.x = fmaf(f, x.x, o.x);
      o.y = fmaf(f, x.y, o.y);
      o.z = fmaf(f, x.z, o.z);
      o.w = fmaf(f, x.w, o.w);
    }
    const int q_head = kv_head * group + h;
    if (to_ws) {
      const int64_t wrow = (static_cast<int64_t>(seq) * p.num_q_heads + q_head) * p.ws_partitions + row;
      *reinterpret_cast<float4*>(p.tmp_out + wrow * D + d) = o;
      if (d == 0) {
        p.max_logits[wrow] = head[h] * kLn2;
        p.exp_sums[wrow] = head[kMaxGroup + h];
      }
    }
    if (to_out) {
      T* dst = static_cast<T*>(p.out) + seq * p.out_stride_seq + q_head * p.out_stride_head + d;
      dst[0] = Conv<T>::from_f32(o.x);
      dst[1] = Conv<T>::from_f32(o.y);
      dst[2] = Conv<T>::from_f32(o.z);
      dst[3] = Conv<T>::from_f32(o.w);
    }
  }
}

// Result of partition `part` of the partition kernels.  A
// sequence whose whole length fits in partition 0 needs no merge: its result
// also goes straight to `out` (the merge kernel skips it), while the
// workspace row is still written so the workspace keeps the same contents.
template <typename T, int D, int WARPS, typename Sync>
__device__ __forceinline__ void write_partition_result(const DecodeParams& p, float* red, int seq, int kv_head,
                                                       int part, int seq_len, int tid, int nthreads, Sync sync) {
  const bool to_out = !p.split || (part == 0 && seq_len <= p.partition_size);
  write_merged_result<T, D, WARPS>(p, red, seq, kv_head, part, p.split != 0, to_out, tid, nthreads, sync);
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
