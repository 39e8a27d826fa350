// Exchange and merge of sequence-shard partials over NVLink peer memory, in
// one kernel per GPU (the collective the NCCL all-gather does, without a
// library round trip).  Each GPU holds, in memory every peer can address
// (symmetric allocations), a flag per rank and two receive buffers of
// R partial blocks [n, Hq, D + 4].  Call number e (kept on the device, so a
// captured CUDA graph replays correctly) runs, on every GPU:
//
//   1. push: copy this GPU's partial rows into slot (e % 2, rank) of every
//      GPU's receive buffer (peer stores over NVLink, 16 bytes at a time);
//   2. publish: every CTA counts itself done after a GPU-scope release of its
//      stores; the last one fences at system scope and stores e into this
//      rank's flag on every GPU (release, system scope);
//   3. wait: every CTA spins (bounded by wait_limit_ns of %globaltimer, then
//      it records the give-up in the error word and carries on) until every
//      rank's flag on this GPU has reached e (acquire, system scope);
//   4. merge: the log-sum-exp merge of the R local slots into `out`;
//   5. the last CTA to finish advances the call counter.
//
// Two receive buffers suffice: a GPU can push call e + 1 only after its merge
// of call e, which needed every peer's flag e, which each peer set only after
// its own merge of call e - 1 -- so slot (e + 1) % 2 is no longer read.
// The grid is at most a few CTAs per SM so that every CTA is resident while
// they wait.  No TMA and no multicast: plain 16-byte peer loads and stores.
#pragma once

#include "decode_params.cuh"
#include "dk_ptx.cuh"

namespace dkb {

constexpr int kExchangeThreads = 256;

struct PeerExchangeParams {
  const float* partial;          // this GPU's rows [n, Hq, D + 4]
  float* recv[kMaxPeers];        // every GPU's receive buffers [2][R][n * Hq * (D + 4)]
  uint32_t* flags[kMaxPeers];    // every GPU's flag words [R]
  uint32_t* state;               // this GPU: [0] completed calls, [1] pushers done, [2] mergers done, [3] errors
  void* out;                     // [n, Hq, D] of T, strided
  int64_t out_stride_seq, out_stride_head;
  int64_t block_floats;          // n * Hq * (D + 4)
  int rank, world, num_seqs, num_q_heads;
  unsigned long long wait_limit_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T, int D>
__global__ void __launch_bounds__(kExchangeThreads) peer_exchange_merge_kernel(const PeerExchangeParams p) {
  constexpr int ROW = D + 4;
  constexpr int V = D / 32;
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  const int tid = threadIdx.x;
  // Launched as a programmatic dependent of the decode that wrote `partial`:
  // scheduled while it drains, everything below waits for its completion.
  pdl_wait_primary();
  if (tid == 0) s_epoch = p.state[0] + 1;  // nothing advances state[0] before every CTA has merged
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = static_cast<int>(e & 1u);

  // 1. push this GPU's rows into slot (par, rank) of every GPU
  const int64_t n4 = p.block_floats / 4;
  const float4* src = reinterpret_cast<const float4*>(p.partial);
  const int64_t slot = (static_cast<int64_t>(par) * p.world + p.rank) * p.block_floats;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kExchangeThreads + tid; i < n4;
       i += static_cast<int64_t>(gridDim.x) * kExchangeThreads) {
    const float4 v = src[i];
    for (int r = 0; r < p.world; ++r) reinterpret_cast<float4*>(p.recv[r] + slot)[i] = v;
  }
  // 2. publish: the last CTA to finish pushing sets this rank's flag everywhere
#ifndef DK_PEER_FENCE_EACH_THREAD
  // The CTA barrier orders every thread's stores before thread 0's
  // GPU-scope release; the last CTA acquires all of them through the counter
  // and its system-scope release of the flags is cumulative over them.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&p.state[1], 1u) == gridDim.x - 1;
  }
#else
  __threadfence_system();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&p.state[1], 1u) == gridDim.x - 1;
#endif
  __syncthreads();
  if (s_last) {
    if (tid == 0) __threadfence_system();
    __syncthreads();
    if (tid < p.world) st_release_sys(p.flags[tid] + p.rank, e);
    if (tid == 0) p.state[1] = 0;
  }
  // 3. wait for every rank's flag on this GPU
  if (tid == 0) {
    const unsigned long long t0 = global_timer_ns();
    for (int r = 0; r < p.world; ++r) {
      while (static_cast<int32_t>(ld_acquire_sys(p.flags[p.rank] + r) - e) < 0) {
        if (global_timer_ns() - t0 > p.wait_limit_ns) {
          atomicAdd(&p.state[3], 1u);
          break;
        }
      }
    }
  }
  __syncthreads();

  // 4. merge the R slots, one warp per (seq, q_head)
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const float* base = p.recv[p.rank] + static_cast<int64_t>(par) * p.world * p.block_floats;
  const int64_t pairs = static_cast<int64_t>(p.num_seqs) * p.num_q_heads;
  for (int64_t pair = static_cast<int64_t>(blockIdx.x) * (kExchangeThreads / 32) + warp; pair < pairs;
       pair += static_cast<int64_t>(gridDim.x) * (kExchangeThreads / 32)) {
    const float* rows = base + pair * ROW;
    float m = -INFINITY;
    for (int r = lane; r < p.world; r += 32) m = fmaxf(m, __ldcg(rows + r * p.block_floats + D));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float acc[V];
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = 0.0f;
    float sum = 0.0f;
    if (m != -INFINITY) {
      for (int r = 0; r < p.world; ++r) {
        const float* row = rows + r * p.block_floats;
        const float w = fast_exp2((__ldcg(row + D) - m) * kLog2e);
        sum += w;
#pragma unroll
        for (int j = 0; j < V; ++j) acc[j] = fmaf(w, __ldcg(row + lane * V + j), acc[j]);
      }
    }
    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
    const int seq = static_cast<int>(pair / p.num_q_heads);
    const int q_head = static_cast<int>(pair - static_cast<int64_t>(seq) * p.num_q_heads);
    T* dst = static_cast<T*>(p.out) + seq * p.out_stride_seq + q_head * p.out_stride_head + lane * V;
#pragma unroll
    for (int j = 0; j < V; ++j) dst[j] = Conv<T>::from_f32(acc[j] * inv);
  }
  // 5. the last CTA to finish advances the call counter
  __syncthreads();
  if (tid == 0 && atomicAdd(&p.state[2], 1u) == gridDim.x - 1) {
    p.state[2] = 0;
    p.state[0] = e;
  }
}

// All-gather of KV-head shards over NVLink peer memory, one kernel per GPU:
// rank r holds the attention output of query heads [r * hpr, (r + 1) * hpr)
// ([n, hpr, D], strided) and every rank needs all heads [n, Hq, D].  The same
// protocol as peer_exchange_merge_kernel, with a copy instead of the merge:
//
//   1. push: this rank's rows into slot (e % 2) of every rank's receive
//      buffer [2][n, Hq, D] at heads [rank * hpr, ...) (16-byte peer stores);
//   2. publish: the last CTA to finish pushing fences at system scope and
//      stores e into this rank's flag on every GPU (release, system scope);
//   3. wait: every CTA waits (bounded by wait_limit_ns; a give-up is counted
//      in the error word) until every rank's flag on this GPU reached e;
//   4. copy the complete slot into `out` (any seq / head strides);
//   5. the last CTA to finish advances the call counter.
//
// Slot (e + 1) % 2 is free when a peer pushes call e + 1 into it for the same
// reason as in the exchange: its last reader, this GPU's copy of call e - 1,
// finished before this GPU published e.  Elements move as opaque 16-bit
// values in 16-byte chunks (rows of D = 64, 128 or 256 elements).
struct PeerGatherParams {
  const uint16_t* local;  // this rank's heads [n, hpr, D]
  int64_t local_stride_seq, local_stride_head;
  uint16_t* recv[kMaxPeers];  // every rank's receive buffers [2][n, Hq, D]
  uint32_t* flags[kMaxPeers];
  uint32_t* state;  // this GPU: [0] completed calls, [1] pushers done, [2] copiers done, [3] errors
  uint16_t* out;    // [n, Hq, D]
  int64_t out_stride_seq, out_stride_head;
  int64_t slot_elems;  // n * Hq * D
  int rank, world, num_seqs, num_q_heads, heads_per_rank, head_dim;
  unsigned long long wait_limit_ns;
};

__global__ void __launch_bounds__(kExchangeThreads) peer_gather_kernel(const PeerGatherParams p) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  const int tid = threadIdx.x;
  // Launched as a programmatic dependent of the decode whose output rows it
  // gathers (or pushed into the slots): everything below waits for it.
  pdl_wait_primary();
  if (tid == 0) s_epoch = p.state[0] + 1;  // nothing advances state[0] before every CTA has copied
  __syncthreads();
  const uint32_t e = s_epoch;
  const int64_t par_off = static_cast<int64_t>(e & 1u) * p.slot_elems;
  const int chunks = p.head_dim >> 3;  // 16-byte chunks per row
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kExchangeThreads;

  // 1. push this rank's rows into slot (e % 2) of every rank (none when the
  //    decode's output stores already did: local == nullptr)
  const int64_t mine = p.local == nullptr ? 0 : static_cast<int64_t>(p.num_seqs) * p.heads_per_rank * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kExchangeThreads + tid; i < mine; i += stride) {
    const int64_t row = i / chunks;
    const int c = static_cast<int>(i - row * chunks);
    const int64_t seq = row / p.heads_per_rank;
    const int h = static_cast<int>(row - seq * p.heads_per_rank);
    const uint4 v = *reinterpret_cast<const uint4*>(p.local + seq * p.local_stride_seq + h * p.local_stride_head + c * 8);
    const int64_t dst = par_off + (seq * p.num_q_heads + p.rank * p.heads_per_rank + h) * p.head_dim + c * 8;
    for (int r = 0; r < p.world; ++r) *reinterpret_cast<uint4*>(p.recv[r] + dst) = v;
  }
  // 2. publish: the last CTA to finish pushing sets this rank's flag everywhere
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&p.state[1], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    if (tid == 0) __threadfence_system();
    __syncthreads();
    if (tid < p.world) st_release_sys(p.flags[tid] + p.rank, e);
    if (tid == 0) p.state[1] = 0;
  }
  // 3. wait for every rank's flag on this GPU
  if (tid == 0) {
    const unsigned long long t0 = global_timer_ns();
    for (int r = 0; r < p.world; ++r) {
      while (static_cast<int32_t>(ld_acquire_sys(p.flags[p.rank] + r) - e) < 0) {
        if (global_timer_ns() - t0 > p.wait_limit_ns) {
          atomicAdd(&p.state[3], 1u);
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. copy the gathered slot into out
  const uint16_t* slot = p.recv[p.rank] + par_off;
  const int64_t all = static_cast<int64_t>(p.num_seqs) * p.num_q_heads * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kExchangeThreads + tid; i < all; i += stride) {
    const int64_t row = i / chunks;
    const int c = static_cast<int>(i - row * chunks);
    const int64_t seq = row / p.num_q_heads;
    const int h = static_cast<int>(row - seq * p.num_q_heads);
    const int4 v = __ldcg(reinterpret_cast<const int4*>(slot + row * p.head_dim + c * 8));  // peers wrote it
    *reinterpret_cast<int4*>(p.out + seq * p.out_stride_seq + h * p.out_stride_head + c * 8) = v;
  }
  // 5. the last CTA to finish advances the call counter
  __syncthreads();
  if (tid == 0 && atomicAdd(&p.state[2], 1u) == gridDim.x - 1) {
    p.state[2] = 0;
    p.state[0] = e;
  }
}

}  // namespace dkb
