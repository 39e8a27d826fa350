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

// Final result of (seq, q_head), columns d..d+3, already normalised.  In LSE
// mode (p.lse_mode) `out` holds fp32 rows (o, lse, pad) and `lse2` -- the
// log2-domain log-sum-exp of the scaled logits, -inf for an empty sequence --
// is stored as a natural log by the thread that writes d == 0.
template <typename T, int D>
__device__ __forceinline__ void store_out4(const DecodeParams& p, int seq, int q_head, int d, float4 o, float lse2) {
  if (p.peer_world > 0) {  // fused head all-gather: this rank's heads into every rank's receive slot
    // the previous call's gather kernel wrote it: read through L2, after the grid-dependency wait
    const int64_t slot = static_cast<int64_t>((__ldcg(p.peer_state) + 1u) & 1u) * p.peer_slot_elems;
    const int64_t at = slot + (static_cast<int64_t>(seq) * p.peer_q_heads + p.peer_head0 + q_head) * D + d;
    const uint2 v = make_uint2(Conv<T>::pack2(o.x, o.y), Conv<T>::pack2(o.z, o.w));
    for (int r = 0; r < p.peer_world; ++r) *reinterpret_cast<uint2*>(static_cast<T*>(p.peer_recv[r]) + at) = v;
    return;
  }
  if (p.lse_mode) {
    float* row = static_cast<float*>(p.out) + seq * p.out_stride_seq + q_head * p.out_stride_head;
    *reinterpret_cast<float4*>(row + d) = o;
    if (d == 0) row[D] = lse2 * kLn2;
    return;
  }
  T* dst = static_cast<T*>(p.out) + seq * p.out_stride_seq + q_head * p.out_stride_head + d;
  dst[0] = Conv<T>::from_f32(o.x);
  dst[1] = Conv<T>::from_f32(o.y);
  dst[2] = Conv<T>::from_f32(o.z);
  dst[3] = Conv<T>::from_f32(o.w);
}

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
    const float inv = p.v_scale / den;  // v_scale: V dequantisation factor (1 for 16-bit caches)
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
    if (to_out) store_out4<T, D>(p, seq, q_head, d, o, head[h] + __log2f(head[kMaxGroup + h]));
  }
}

// Shared state of the single-launch merge, one copy per CTA for every caller
// (a variable inside a function templated on the barrier type would exist
// once per instantiation, and the producer and consumer warps pass different
// lambdas): [0] the "this partition merges" flag, then per head of the group
// the max logit (log2 units) and 1 / exp-sum.
__device__ __forceinline__ float* merge_shared() {
  __shared__ float s_merge[1 + 2 * kMaxGroup];
  return s_merge;
}

// Counter increment with release (this CTA's prior global writes, ordered
// before it by the CTA barrier, are visible first) and acquire (the other
// partitions' writes are visible after it) semantics at GPU scope.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Single-launch merge (p.merge_counters set): every live partition of
// (seq, kv_head) publishes its workspace rows with one counter increment
// (after the CTA barrier, release semantics); the partition that brings the
// count to the number of live partitions merges the group's rows into `out`
// and resets the counter to 0 for the next call.  No thread waits on another
// CTA.  The merge keeps every load independent: per head (one warp, a row
// per lane) the max logit and exp-sum, then every thread sums w_i * o_i for
// 4 output columns, 8 rows in flight at a time.  Rows are read through L2
// (ld.global.cg): other CTAs wrote them.
template <typename T, int D, typename Sync>
__device__ __forceinline__ void merge_if_last(const DecodeParams& p, int seq, int kv_head, int live, int tid,
                                              int nthreads, Sync sync) {
  float* sh = merge_shared();
  sync();  // every thread's workspace stores precede the release below
  if (tid == 0) {
    int* ctr = p.merge_counters + static_cast<int64_t>(seq) * p.num_kv_heads + kv_head;
    const int last = atomic_add_acq_rel_gpu(ctr, 1) == live - 1;
    if (last) *ctr = 0;  // every live partition has counted: nothing else touches it in this call
    sh[0] = last ? 1.0f : 0.0f;
  }
  sync();
  if (sh[0] == 0.0f) return;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int group = p.group;
  const int64_t head0 = static_cast<int64_t>(seq) * p.num_q_heads + kv_head * group;  // first q-head of the group
  for (int h = warp; h < group; h += nthreads >> 5) {
    const float* ml = p.max_logits + (head0 + h) * p.ws_partitions;
    const float* es = p.exp_sums + (head0 + h) * p.ws_partitions;
    float m = -INFINITY, w = 0.0f;  // lane-local running (max, sum) over rows lane, lane + 32, ...
    for (int i = lane; i < live; i += 32) {
      const float mi = __ldcg(ml + i) * kLog2e;
      const float si = __ldcg(es + i);
      const float mn = fmaxf(m, mi);
      w = fmaf(w, fast_exp2(m - mn), si * fast_exp2(mi - mn));
      m = mn;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m, o);
      const float wo = __shfl_xor_sync(0xffffffffu, w, o);
      const float mn = fmaxf(m, mo);
      w = (mn == -INFINITY) ? 0.0f : w * fast_exp2(m - mn) + wo * fast_exp2(mo - mn);
      m = mn;
    }
    if (lane == 0) {
      sh[1 + h] = m;
      sh[1 + kMaxGroup + h] = 1.0f / w;
    }
  }
  sync();
  constexpr int Q = D / 4;
  constexpr int kBatch = 8;
  for (int idx = tid; idx < group * Q; idx += nthreads) {
    const int h = idx / Q;
    const int d = (idx - h * Q) * 4;
    const int64_t row0 = (head0 + h) * p.ws_partitions;
    const float m2 = sh[1 + h];
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int i0 = 0; i0 < live; i0 += kBatch) {
      float wi[kBatch];
      float4 x[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        wi[k] = 0.0f;
        x[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i0 + k < live) {
          const int64_t r = row0 + i0 + k;
          wi[k] = __ldcg(p.exp_sums + r) * fast_exp2(fmaf(__ldcg(p.max_logits + r), kLog2e, -m2));
          x[k] = __ldcg(reinterpret_cast<const float4*>(p.tmp_out + r * D + d));
        }
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        acc.x = fmaf(wi[k], x[k].x, acc.x);
        acc.y = fmaf(wi[k], x[k].y, acc.y);
        acc.z = fmaf(wi[k], x[k].z, acc.z);
        acc.w = fmaf(wi[k], x[k].w, acc.w);
      }
    }
    const float inv = sh[1 + kMaxGroup + h];
    store_out4<T, D>(p, seq, kv_head * group + h, d,
                     make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv), m2 - __log2f(inv));
  }
}

// Result of partition `part` (of `partition_size` tokens, the size in force
// for this launch) of the partition kernels.  A sequence whose whole length
// fits in partition 0 needs no merge: its result also goes straight to `out`
// (the merge kernel skips it), while the workspace row is still written so
// the workspace keeps the same contents.
template <typename T, int D, int WARPS, typename Sync>
__device__ __forceinline__ void write_partition_result(const DecodeParams& p, float* red, int seq, int kv_head,
                                                       int part, int seq_len, int partition_size, int tid,
                                                       int nthreads, Sync sync) {
  const bool to_out = !p.split || (part == 0 && seq_len <= partition_size);
  write_merged_result<T, D, WARPS>(p, red, seq, kv_head, part, p.split != 0, to_out, tid, nthreads, sync);
  if (p.merge_counters != nullptr && !to_out)
    merge_if_last<T, D>(p, seq, kv_head, (seq_len + partition_size - 1) / partition_size, tid, nthreads, sync);
}

// Empty sequences get exact zeros from the partition kernel when no merge
// kernel runs after it (single pass, or the single-launch merge).
__device__ __forceinline__ bool partition_writes_zeros(const DecodeParams& p, int part, int seq_len) {
  return !p.split || (p.merge_counters != nullptr && part == 0 && seq_len <= 0);
}

// Zeros for the group's query heads of an empty sequence (single-pass path),
// matching csrc/paged_attention.cuh:91-105.
template <typename T, int D>
__device__ __forceinline__ void write_zero_output(const DecodeParams& p, int seq, int kv_head, int tid, int nthreads) {
  constexpr int Q = D / 4;
  for (int idx = tid; idx < p.group * Q; idx += nthreads) {
    const int h = idx / Q;
    store_out4<T, D>(p, seq, kv_head * p.group + h, (idx - h * Q) * 4, make_float4(0.0f, 0.0f, 0.0f, 0.0f), -INFINITY);
  }
}

}  // namespace dkb
