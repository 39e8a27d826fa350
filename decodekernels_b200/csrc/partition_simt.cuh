// Partition kernel, CUDA-core path for caches the TMA path cannot describe
// (block sizes that are not a power-of-two divisor or multiple of 64 tokens,
// strides or base pointers that are not 16-byte aligned).  It accepts exactly
// what DecodeKernels accepts (csrc/ops.cu:72-79: strides a multiple of
// head_dim / 32 elements, pointers aligned to head_dim / 16 bytes) and writes
// the same outputs and workspace rows as the fast path.
//
// One CTA of 4 warps per (partition, kv_head, seq).  Warp w takes tokens
// pstart + w, pstart + w + 4, ...; lane i holds head_dim / 32 contiguous
// elements of each K/V row (one vector load), the group's query vectors stay
// in registers, and each warp keeps an online softmax per query head, so K
// and V are read in one pass.  The warps merge in partition_epilogue.cuh.
#pragma once

#include "decode_params.cuh"
#include "dk_ptx.cuh"
#include "partition_epilogue.cuh"

namespace dkb {

template <typename T, int N>
struct alignas(sizeof(T) * N) VecT {
  T v[N];
};

template <int D>
struct SimtConfig {
  static constexpr int kWarps = kSimtThreads / 32;
  static constexpr int kSmemBytes = RedLayout<D>::floats(kWarps) * 4;
};

// Cache element -> float: the 16-bit types, or e4m3 bytes (exact).
__device__ __forceinline__ float kv_to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float kv_to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float kv_to_f32(uint8_t x) { return e4m3_to_f32(x); }

// KV: cache element type (T, or uint8_t for e4m3 caches, whose k_scale is in
// p.scale_log2 and v_scale in the epilogue).
template <typename T, int D, typename KV = T>
__global__ void __launch_bounds__(kSimtThreads) paged_decode_simt_kernel(const DecodeParams p) {
  constexpr int V = D / 32;
  constexpr int WARPS = kSimtThreads / 32;
  using Vec = VecT<KV, V>;
  extern __shared__ float simt_smem[];

  int part, kv_head, seq;
  cta_coords(p.num_partitions, p.num_kv_heads, part, kv_head, seq);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int group = p.group;

  pdl_wait_primary();
  const int seq_len = min(p.seq_lens[seq], p.max_seq_len);  // lengths above max_seq_len count as max_seq_len
  const int pstart = part * p.partition_size;
  if (pstart >= seq_len) {
    if (partition_writes_zeros(p, part, seq_len)) write_zero_output<T, D>(p, seq, kv_head, threadIdx.x, kSimtThreads);
    pdl_launch_dependents();
    return;
  }
  const int pend = min(pstart + p.partition_size, seq_len);

  float qv[kMaxGroup][V];
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) {
    if (h < group) {
      // q has no alignment requirement (DecodeKernels reads it element-wise)
      const T* qp = static_cast<const T*>(p.q) + seq * p.q_stride_seq + (kv_head * group + h) * p.q_stride_head +
                    lane * V;
#pragma unroll
      for (int j = 0; j < V; ++j) qv[h][j] = Conv<T>::to_f32(qp[j]) * p.scale_log2;
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) qv[h][j] = 0.0f;
    }
  }

  float m[kMaxGroup], l[kMaxGroup], acc[kMaxGroup][V];
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int j = 0; j < V; ++j) acc[h][j] = 0.0f;
  }

  const KV* kc = static_cast<const KV*>(p.k_cache);
  const KV* vc = static_cast<const KV*>(p.v_cache);
  const int* bt = p.block_tables + static_cast<int64_t>(seq) * p.bt_stride;
  for (int t = pstart + warp; t < pend; t += WARPS) {
    const int lb = t / p.block_size;
    const int off = t - lb * p.block_size;
    const int64_t pb = __ldg(bt + lb);
    float kf[V], vf[V];
    if (pb >= 0 && pb < p.num_blocks) {
      const Vec kx = *reinterpret_cast<const Vec*>(kc + pb * p.k_stride_block + off * p.k_stride_token +
                                                   kv_head * p.k_stride_head + lane * V);
      const Vec vx = *reinterpret_cast<const Vec*>(vc + pb * p.v_stride_block + off * p.v_stride_token +
                                                   kv_head * p.v_stride_head + lane * V);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        kf[j] = kv_to_f32(kx.v[j]);
        vf[j] = kv_to_f32(vx.v[j]);
      }
    } else {  // out-of-range block id: zeros, like the TMA path's out-of-bounds fill
#pragma unroll
      for (int j = 0; j < V; ++j) kf[j] = vf[j] = 0.0f;
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
      if (h < group) {
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < V; ++j) s = fmaf(qv[h][j], kf[j], s);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mn = fmaxf(m[h], s);
        const float al = fast_exp2(m[h] - mn);
        const float pr = fast_exp2(s - mn);
        m[h] = mn;
        l[h] = fmaf(l[h], al, pr);
#pragma unroll
        for (int j = 0; j < V; ++j) acc[h][j] = fmaf(acc[h][j], al, pr * vf[j]);
      }
    }
  }
  pdl_launch_dependents();

  using Red = RedLayout<D>;
  constexpr int R = Red::kRow;
  float* red_o = Red::o(simt_smem);
  float* red_m = Red::m(simt_smem, WARPS);
  float* red_l = Red::l(simt_smem, WARPS);
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) {
    if (h < group) {
#pragma unroll
      for (int j = 0; j < V; ++j) red_o[(warp * kMaxGroup + h) * R + lane * V + j] = acc[h][j];
      if (lane == 0) {
        red_m[warp * kMaxGroup + h] = m[h];
        red_l[warp * kMaxGroup + h] = l[h];
      }
    }
  }
  __syncthreads();
  write_partition_result<T, D, WARPS>(p, simt_smem, seq, kv_head, part, seq_len, p.partition_size, threadIdx.x,
                                      kSimtThreads, [] { __syncthreads(); });
}

}  // namespace dkb
