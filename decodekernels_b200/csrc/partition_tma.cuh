// Partition kernel, sm_100a fast path: TMA-staged KV pages + tensor-core math.
//
// One CTA per (partition, kv_head, seq) computes all `group` query heads of
// its KV head, so every K/V byte is read from HBM once (DecodeKernels'
// GQA-aware block, csrc/paged_attention.cuh:73-225, re-designed):
//
// * Warp 4 (producer) reads the partition's block-table slice (32 entries per
//   coalesced load, prefetched one group ahead) and issues, per 64-token tile,
//   one 4-D TMA box per (page, 64-column half) for K and for V into a
//   NSTAGES-deep shared-memory ring.  The tensor maps describe the caches with
//   their real strides, so vLLM's interleaved K|V and FlashInfer NHD/HND views
//   are read in place.  Boxes use the 128-byte swizzle, so the ldmatrix reads
//   below are bank-conflict free.  Block ids outside [0, num_blocks) read
//   zeros (TMA out-of-bounds fill) instead of faulting.
// * Warps 0-3 (consumers) each own 16 tokens of every tile.  S^T = K Q^T on
//   mma.m16n8k16 (M = 16 tokens, N = 8 query heads, K = head_dim), online
//   softmax in registers (the head columns of S^T and of the O^T accumulator
//   live in the same lanes), P^T rebuilt as a B fragment with movmatrix, and
//   O^T += V^T P^T on mma.m16n8k16 with ldmatrix.trans.  fp32 accumulation.
// * A full/empty mbarrier pair per stage couples them; every wait is bounded.
// * The cross-warp merge and the write-out are in partition_epilogue.cuh.
#pragma once

#include "decode_params.cuh"
#include "dk_ptx.cuh"
#include "partition_epilogue.cuh"

namespace dkb {

template <int D, int NSTAGES>
struct TmaConfig {
  static constexpr int kHalves = D / 64;                        // 128-byte column blocks per row
  static constexpr int kHalfBytes = kTileTokens * 128;          // one column block of a tile
  static constexpr int kTileBytes = kHalves * kHalfBytes;       // K (or V) of one tile
  static constexpr int kStageBytes = 2 * kTileBytes;            // K + V
  static constexpr int kSmemBytes = NSTAGES * kStageBytes + 1024;  // + alignment slack
  static_assert(RedLayout<D>::floats(kConsumerWarps) * 4 <= NSTAGES * kStageBytes, "merge scratch must fit");
};

__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
}

template <typename T, int D, int NSTAGES>
__global__ void __launch_bounds__(kTmaThreads) paged_decode_tma_kernel(const __grid_constant__ CUtensorMap k_map,
                                                                       const __grid_constant__ CUtensorMap v_map,
                                                                       const DecodeParams p) {
  using Cfg = TmaConfig<D, NSTAGES>;
  constexpr int MT = D / 16;  // 16-wide blocks of head_dim

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_k[NSTAGES];
  __shared__ __align__(8) uint64_t full_v[NSTAGES];
  __shared__ __align__(8) uint64_t empty_bar[NSTAGES];

  const int part = blockIdx.x;
  const int kv_head = blockIdx.y;
  const int seq = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&full_k[s], 1);
      mbar_init(&full_v[s], 1);
      mbar_init(&empty_bar[s], kConsumerWarps);
    }
    mbar_init_fence();
  }
  if (warp == kConsumerWarps && lane == 0) {
    tma_prefetch_desc(&k_map);
    tma_prefetch_desc(&v_map);
  }
  __syncthreads();

  // Inputs written by the previous kernel in the stream are visible after this.
  pdl_wait_primary();

  const int seq_len = p.seq_lens[seq];
  const int pstart = part * p.partition_size;
  if (pstart >= seq_len) {
    // Empty sequence (single pass writes zeros) or a partition past the end
    // (skipped; the merge kernel reads only live partitions).
    if (!p.split) write_zero_output<T, D>(p, seq, kv_head, threadIdx.x, kTmaThreads);
    pdl_launch_dependents();
    return;
  }
  const int pend = min(pstart + p.partition_size, seq_len);
  const int ntiles = (pend - pstart + kTileTokens - 1) / kTileTokens;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------------ producer
    const int bs = p.block_size;
    const int rows = p.rows_per_op;
    const int lb0 = pstart / bs;
    const int nlb = (pend - 1) / bs - lb0 + 1;  // logical blocks this partition touches
    const int* bt = p.block_tables + static_cast<int64_t>(seq) * p.bt_stride + lb0;
    int cur = (lane < nlb) ? __ldg(bt + lane) : 0;
    int nxt = (32 + lane < nlb) ? __ldg(bt + 32 + lane) : 0;
    int base = 0;
    const uint64_t policy = l2_evict_first_policy();
    const uint32_t box_bytes = static_cast<uint32_t>(rows) * 128u;

    for (int t = 0; t < ntiles; ++t) {
      const int s = t % NSTAGES;
      if (!mbar_wait(&empty_bar[s], ((t / NSTAGES) & 1) ^ 1)) break;
      const int tstart = pstart + t * kTileTokens;
      const int nops = (min(kTileTokens, pend - tstart) + rows - 1) / rows;

      int pbs[kTileTokens / 8];
#pragma unroll
      for (int j = 0; j < kTileTokens / 8; ++j) {
        int pb = 0;
        if (j < nops) {
          const int rel = (tstart + j * rows) / bs - lb0;
          while (rel >= base + 32) {  // warp-uniform
            base += 32;
            cur = nxt;
            nxt = (base + 32 + lane < nlb) ? __ldg(bt + base + 32 + lane) : 0;
          }
          pb = __shfl_sync(0xffffffffu, cur, rel - base);
        }
        pbs[j] = pb;
      }

      if (lane == 0) {
        uint8_t* kdst = smem + s * Cfg::kStageBytes;
        uint8_t* vdst = kdst + Cfg::kTileBytes;
        const uint32_t bytes = static_cast<uint32_t>(nops * Cfg::kHalves) * box_bytes;
        mbar_arrive_expect_tx(&full_k[s], bytes);
        mbar_arrive_expect_tx(&full_v[s], bytes);
#pragma unroll
        for (int kv = 0; kv < 2; ++kv) {
          const CUtensorMap* map = kv == 0 ? &k_map : &v_map;
          uint8_t* dst = kv == 0 ? kdst : vdst;
          uint64_t* bar = kv == 0 ? &full_k[s] : &full_v[s];
#pragma unroll
          for (int j = 0; j < kTileTokens / 8; ++j) {
            if (j < nops) {
              const int tok = tstart + j * rows;
              const int off = tok - (tok / bs) * bs;
              const int pb = pbs[j];
              const int c1 = p.slot_head == 1 ? kv_head : (p.slot_tok == 1 ? off : pb);
              const int c2 = p.slot_head == 2 ? kv_head : (p.slot_tok == 2 ? off : pb);
              const int c3 = p.slot_head == 3 ? kv_head : (p.slot_tok == 3 ? off : pb);
#pragma unroll
              for (int h = 0; h < Cfg::kHalves; ++h) {
                tma_load_4d(dst + h * Cfg::kHalfBytes + j * box_bytes, map, h * 64, c1, c2, c3, bar, policy);
              }
            }
          }
        }
      }
      __syncwarp();
    }
    pdl_launch_dependents();
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int group = p.group;
  const int qn = lane >> 2;  // query head of this lane's B-fragment column
  uint32_t qf[MT][2];
  {
    const uint16_t* qrow = static_cast<const uint16_t*>(p.q) + static_cast<int64_t>(seq) * p.q_stride_seq +
                           static_cast<int64_t>(kv_head * group + qn) * p.q_stride_head;
#pragma unroll
    for (int kk = 0; kk < MT; ++kk) {
      const int d0 = kk * 16 + 2 * (lane & 3);
      if (qn < group) {
        qf[kk][0] = pack_raw16(qrow[d0], qrow[d0 + 1]);
        qf[kk][1] = pack_raw16(qrow[d0 + 8], qrow[d0 + 9]);
      } else {
        qf[kk][0] = 0u;
        qf[kk][1] = 0u;
      }
    }
  }

  float m0 = -INFINITY, m1 = -INFINITY;  // running max of columns c0, c0+1 (log2 units)
  float l0 = 0.0f, l1 = 0.0f;            // this lane's share of the exp-sums
  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[mt][j] = 0.0f;
  }

  const uint32_t smem_base = smem_u32(smem);
  const int r0 = warp * kSubTokens;                                // first tile row of this warp
  const int k_row = r0 + (lane & 7) + (((lane >> 3) & 1) << 3);    // ldmatrix row (K as A, row-major)
  const int k_chunk = lane >> 4;                                   // 0: k 0-7, 1: k 8-15
  const int v_row = r0 + (lane & 7) + ((lane >> 4) << 3);          // ldmatrix.trans row (V^T as A)
  const int v_chunk = (lane >> 3) & 1;                             // 0: d 0-7, 1: d 8-15

  for (int t = 0; t < ntiles; ++t) {
    const int s = t % NSTAGES;
    const uint32_t parity = (t / NSTAGES) & 1;
    const int sub0 = pstart + t * kTileTokens + r0;  // first token of this warp's 16
    if (sub0 < pend) {
      if (!mbar_wait(&full_k[s], parity)) break;
      const uint32_t kb = smem_base + s * Cfg::kStageBytes;

      // S^T[16 tokens][8 heads] = K Q^T, two accumulator chains
      float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      float sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int kk = 0; kk < MT; ++kk) {
        const int chunk = ((kk & 3) << 1) + k_chunk;
        const uint32_t addr = kb + (kk >> 2) * Cfg::kHalfBytes + k_row * 128 + ((chunk ^ (k_row & 7)) << 4);
        uint32_t a[4];
        ldmatrix_x4(a, addr);
        if (kk & 1)
          Mma<T>::run(sb, a, qf[kk][0], qf[kk][1]);
        else
          Mma<T>::run(sa, a, qf[kk][0], qf[kk][1]);
      }
      float sc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[i] = (sa[i] + sb[i]) * p.scale_log2;
      const int tok_a = sub0 + (lane >> 2);  // token of sc[0], sc[1]; sc[2], sc[3] are 8 later
      if (tok_a >= pend) sc[0] = sc[1] = -INFINITY;
      if (tok_a + 8 >= pend) sc[2] = sc[3] = -INFINITY;

      // online softmax over the 16 tokens (column max across the 8 lanes of a column)
      float mx0 = fmaxf(sc[0], sc[2]);
      float mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0);
      const float mn1 = fmaxf(m1, mx1);
      const float al0 = fast_exp2(m0 - mn0);
      const float al1 = fast_exp2(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      const float p0 = fast_exp2(sc[0] - mn0);
      const float p1 = fast_exp2(sc[1] - mn1);
      const float p2 = fast_exp2(sc[2] - mn0);
      const float p3 = fast_exp2(sc[3] - mn1);
      l0 = fmaf(l0, al0, p0 + p2);
      l1 = fmaf(l1, al1, p1 + p3);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        acc[mt][0] *= al0;
        acc[mt][1] *= al1;
        acc[mt][2] *= al0;
        acc[mt][3] *= al1;
      }
      // P^T as the B fragment of O^T += V^T P^T
      const uint32_t pb0 = movmatrix_trans(Conv<T>::pack2(p0, p1));
      const uint32_t pb1 = movmatrix_trans(Conv<T>::pack2(p2, p3));

      if (!mbar_wait(&full_v[s], parity)) break;
      const uint32_t vb = kb + Cfg::kTileBytes;
      if (sub0 + kSubTokens > pend) {
        // Rows of tokens >= pend hold whatever the page (or an earlier tile)
        // left there; P is 0 for them but 0 * NaN is NaN, so clear them.
        const int first_bad = pend - (sub0 - r0);
        for (int i = lane; i < kSubTokens * Cfg::kHalves * 8; i += 32) {
          const int row = r0 + i / (Cfg::kHalves * 8);
          const int rem = i % (Cfg::kHalves * 8);
          if (row >= first_bad) st_shared_zero16(vb + (rem >> 3) * Cfg::kHalfBytes + row * 128 + ((rem & 7) << 4));
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int chunk = ((mt & 3) << 1) + v_chunk;
        const uint32_t addr = vb + (mt >> 2) * Cfg::kHalfBytes + v_row * 128 + ((chunk ^ (v_row & 7)) << 4);
        uint32_t a[4];
        ldmatrix_x4_trans(a, addr);
        Mma<T>::run(acc[mt], a, pb0, pb1);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  }
  pdl_launch_dependents();

  // Full exp-sums per column: add the 8 lanes that share it.
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }

  // Every tile's TMA writes have landed (warp 0 waits on every tile), so the
  // ring can be reused for the cross-warp merge once all consumers are here.
  named_bar_sync(1, kConsumerWarps * 32);
  constexpr int R = RedLayout<D>::kRow;
  float* red_o = reinterpret_cast<float*>(smem);
  float* red_m = red_o + kConsumerWarps * kMaxGroup * R;
  float* red_l = red_m + kConsumerWarps * kMaxGroup;
  const int c0 = 2 * (lane & 3);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int h = c0 + (j & 1);
      const int d = mt * 16 + (lane >> 2) + ((j >> 1) << 3);
      if (h < group) red_o[(warp * kMaxGroup + h) * R + d] = acc[mt][j];
    }
  }
  if (lane < 4) {
    red_m[warp * kMaxGroup + c0] = m0;
    red_m[warp * kMaxGroup + c0 + 1] = m1;
    red_l[warp * kMaxGroup + c0] = l0;
    red_l[warp * kMaxGroup + c0 + 1] = l1;
  }
  named_bar_sync(1, kConsumerWarps * 32);
  write_partition_result<T, D, kConsumerWarps>(p, red_o, red_m, red_l, seq, kv_head, part, threadIdx.x,
                                               kConsumerWarps * 32);
}

}  // namespace dkb
