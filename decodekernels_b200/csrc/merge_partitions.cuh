// Log-sum-exp merge of split-K partitions (DecodeKernels'
// paged_attention_reduce_kernel, csrc/paged_attention.cuh:227-269):
//   M = max_i m_i,  w_i = s_i exp(m_i - M),  out = sum_i w_i o_i / sum_i w_i
// over the live partitions num_parts = min(ceil(L / partition_size), P), with
// the partition size the partition kernel used (fit_partition_size's choice
// when the planner left it to the device);
// zeros when L <= 0.  Sequences with a single live partition were already
// written to `out` by the partition kernel and are skipped here.
//
// One CTA of 8 warps per (query head, sequence).  Warp w folds partitions
// w, w+8, ... in one pass with a running max (rescaling its partial sum when
// the max grows), each lane holding head_dim / 32 consecutive floats of a
// partial output (one 8/16/32-byte load per partition, unrolled so several
// are in flight); the eight (max, sum, output) states are then combined
// through shared memory.  Launched with programmatic dependent launch: the
// CTAs start while the partition kernel drains and wait for its results in
// griddepcontrol.wait.
#pragma once

#include "decode_params.cuh"
#include "dk_ptx.cuh"
#include "partition_epilogue.cuh"

namespace dkb {

template <int N>
struct alignas(4 * N) F32Vec {
  float v[N];
};

constexpr int kMergeWarps = kMergeThreads / 32;

// Fold workspace rows [0, num_rows) of (seq, q_head) into `out` (all threads
// of the CTA take part).
template <typename T, int D>
__device__ __forceinline__ void merge_rows(const DecodeParams& p, int seq, int q_head, int num_rows) {
  constexpr int V = D / 32;
  using Vec = F32Vec<V>;
  __shared__ float red[kMergeWarps][D];
  __shared__ float wmax[kMergeWarps];
  __shared__ float wsum[kMergeWarps];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row0 = (static_cast<int64_t>(seq) * p.num_q_heads + q_head) * p.ws_partitions;
  const float* ml = p.max_logits + row0;
  const float* es = p.exp_sums + row0;
  const float* tmp = p.tmp_out + row0 * D + lane * V;

  // running state in log2 units: acc = sum_i s_i 2^(m_i - m) o_i, sum = sum_i s_i 2^(m_i - m)
  float m = -INFINITY, sum = 0.0f;
  float acc[V];
#pragma unroll
  for (int j = 0; j < V; ++j) acc[j] = 0.0f;
#pragma unroll 4
  for (int i = warp; i < num_rows; i += kMergeWarps) {
    const float mi = ml[i] * kLog2e;
    const float si = es[i];
    const Vec x = *reinterpret_cast<const Vec*>(tmp + static_cast<int64_t>(i) * D);
    const float mn = fmaxf(m, mi);
    const float keep = fast_exp2(m - mn);  // 0 on the first row
    const float w = si * fast_exp2(mi - mn);
    m = mn;
    sum = fmaf(sum, keep, w);
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = fmaf(acc[j], keep, w * x.v[j]);
  }
#pragma unroll
  for (int j = 0; j < V; ++j) red[warp][lane * V + j] = acc[j];
  if (lane == 0) {
    wmax[warp] = m;
    wsum[warp] = sum;
  }
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kMergeWarps; ++w) M = fmaxf(M, wmax[w]);
  float f[kMergeWarps];
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < kMergeWarps; ++w) {
    f[w] = fast_exp2(wmax[w] - M);  // 0 for warps without rows
    total = fmaf(f[w], wsum[w], total);
  }
  const float inv = 1.0f / total;
  const float lse2 = M + __log2f(total);
  for (int d = threadIdx.x * 4; d < D; d += kMergeThreads * 4) {
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[j] = 0.0f;
#pragma unroll
      for (int w = 0; w < kMergeWarps; ++w) o[j] = fmaf(f[w], red[w][d + j], o[j]);
    }
    store_out4<T, D>(p, seq, q_head, d, make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv), lse2);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kMergeThreads) merge_partitions_kernel(const DecodeParams p) {
  const int q_head = blockIdx.x;
  const int seq = blockIdx.y;
  pdl_wait_primary();
  // A fitted size: the partition kernel's choice, which its CTA 0 left in the
  // reserved workspace slot (fit_size_slot).
  const int ps = p.fit_slots > 0 ? __float_as_int(__ldcg(fit_size_slot(p))) : p.partition_size;
  const int seq_len = min(p.seq_lens[seq], p.max_seq_len);  // lengths above max_seq_len count as max_seq_len
  if (seq_len <= 0) {
    for (int d = threadIdx.x * 4; d < D; d += kMergeThreads * 4)
      store_out4<T, D>(p, seq, q_head, d, make_float4(0.0f, 0.0f, 0.0f, 0.0f), -INFINITY);
    return;
  }
  const int num_parts = min((seq_len + ps - 1) / ps, p.num_partitions);
  if (num_parts <= 1) return;  // written by the partition kernel
  merge_rows<T, D>(p, seq, q_head, num_parts);
}

// Merge of attention partials computed over disjoint token ranges (for
// example the sequence shards of several GPUs): rows (o, lse, pad) of
// `num_parts` fp32 buffers [n, Hq, D + 4] spaced `part_stride` floats apart,
//   M = max_r lse_r,  w_r = exp(lse_r - M),  out = sum_r w_r o_r / sum_r w_r,
// lse = M + log(sum_r w_r); zeros (and lse = -inf) when every part is empty.
// One warp per (seq, q_head), lane holding D / 32 consecutive columns.
struct LseMergeParams {
  const float* parts;
  int64_t part_stride;
  void* out;  // T [n, Hq, D] strided, or fp32 rows (o, lse, pad) when out_lse
  int64_t out_stride_seq, out_stride_head;
  int num_parts, num_seqs, num_q_heads;
  int out_lse;
};

constexpr int kLseMergeThreads = 128;

template <typename T, int D>
__global__ void __launch_bounds__(kLseMergeThreads) merge_lse_kernel(const LseMergeParams p) {
  constexpr int V = D / 32;
  constexpr int ROW = D + 4;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t pair = static_cast<int64_t>(blockIdx.x) * (kLseMergeThreads / 32) + warp;
  if (pair >= static_cast<int64_t>(p.num_seqs) * p.num_q_heads) return;
  const int seq = static_cast<int>(pair / p.num_q_heads);
  const int q_head = static_cast<int>(pair - static_cast<int64_t>(seq) * p.num_q_heads);
  const float* base = p.parts + pair * ROW;
  float m = -INFINITY;
  for (int r = lane; r < p.num_parts; r += 32) m = fmaxf(m, base[r * p.part_stride + D]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float acc[V];
#pragma unroll
  for (int j = 0; j < V; ++j) acc[j] = 0.0f;
  float sum = 0.0f;
  if (m != -INFINITY) {
    for (int r = 0; r < p.num_parts; ++r) {
      const float* row = base + r * p.part_stride;
      const float w = fast_exp2((row[D] - m) * kLog2e);  // 0 for empty parts (lse = -inf)
      sum += w;
#pragma unroll
      for (int j = 0; j < V; ++j) acc[j] = fmaf(w, row[lane * V + j], acc[j]);
    }
  }
  const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
  if (p.out_lse) {
    float* row = static_cast<float*>(p.out) + seq * p.out_stride_seq + q_head * p.out_stride_head;
#pragma unroll
    for (int j = 0; j < V; ++j) row[lane * V + j] = acc[j] * inv;
    if (lane == 0) row[D] = sum > 0.0f ? m + __logf(sum) : -INFINITY;
    return;
  }
  T* dst = static_cast<T*>(p.out) + seq * p.out_stride_seq + q_head * p.out_stride_head + lane * V;
#pragma unroll
  for (int j = 0; j < V; ++j) dst[j] = Conv<T>::from_f32(acc[j] * inv);
}

}  // namespace dkb
