// Partition kernel, sm_100a fast path: TMA-staged KV pages + tensor-core math.
//
// One CTA per (partition, kv_head, seq) computes all `group` query heads of
// its KV head, so every K/V byte is read from HBM once (DecodeKernels'
// GQA-aware block, csrc/paged_attention.cuh:73-225, re-designed):
//
// * Warp WARPS (producer) reads the partition's block-table slice (32 entries per
//   coalesced load, the next group prefetched) and, per tile, issues
//   ONE 5-D TMA box per page for K and one for V -- or a single box for both
//   when the cache is vLLM's interleaved K|V buffer -- into an NSTAGES-deep
//   shared-memory ring.  The tensor maps are (64 columns, token, 64-column
//   block, head, block) with the caches' real strides, so the vLLM and
//   FlashInfer NHD/HND views are read in place, and a box lands as
//   [column block][page row][128 B], 128-byte swizzled.  Block-size arithmetic
//   is shifts (power-of-two block sizes only on this path).  Block ids outside
//   [0, num_blocks) read zeros (TMA out-of-bounds fill) instead of faulting.
// * Warps 0..WARPS-1 (consumers) each own 16 tokens of every tile.  S^T = K Q^T on
//   mma.m16n8k16 (M = 16 tokens, N = 8 query heads, K = head_dim), online
//   softmax in registers (the head columns of S^T and of the O^T accumulator
//   live in the same lanes), P^T rebuilt as a B fragment with movmatrix, and
//   O^T += V^T P^T on mma.m16n8k16 with ldmatrix.trans.  fp32 accumulation.
//   Every 8-row ldmatrix group lies inside one page, whose rows carry distinct
//   swizzle phases, so the shared-memory reads are bank-conflict free.
// * A full/empty mbarrier pair per stage couples them; every wait is bounded.
// * The cross-warp merge and the write-out are in partition_epilogue.cuh.
#pragma once

#include "decode_params.cuh"
#include "dk_ptx.cuh"
#include "partition_epilogue.cuh"

namespace dkb {

// WARPS consumer warps of 16 tokens each make a tile of 16 * WARPS tokens
// (64 for head_dim <= 128, 32 for head_dim 256 so that several CTAs fit on
// an SM); a tile divides the 64-token partition granularity.
template <int D, int NSTAGES, int WARPS>
struct TmaConfig {
  static constexpr int kWarps = WARPS;
  static constexpr int kTile = kSubTokens * WARPS;                 // tokens per pipeline stage
  static constexpr int kThreads = (WARPS + 1) * 32;                // + one TMA producer warp
  static constexpr int kHalves = D / 64;                           // 128-byte column blocks per row
  static constexpr int kTileBytes = kHalves * kTile * 128;         // K (or V) of one tile
  static constexpr int kStageBytes = 2 * kTileBytes;               // K + V
  static constexpr int kSmemBytes = NSTAGES * kStageBytes + 1024;  // + alignment slack
  static_assert(kTileTokens % kTile == 0, "a tile must divide the partition granularity");
  static_assert(RedLayout<D>::floats(WARPS) * 4 <= NSTAGES * kStageBytes, "merge scratch must fit");
};

__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
}

// Stage layout: page-major.  Page j of a tile (rows = min(block_size, tile)
// token rows) occupies kPage = 2 * kHalves * rows * 128 bytes: the K column
// blocks [h][row][128 B] followed by the V column blocks.
template <typename T, int D, int NSTAGES, int WARPS>
__global__ void __launch_bounds__((WARPS + 1) * 32) paged_decode_tma_kernel(const __grid_constant__ CUtensorMap k_map,
                                                                       const __grid_constant__ CUtensorMap v_map,
                                                                       const DecodeParams p) {
  using Cfg = TmaConfig<D, NSTAGES, WARPS>;
  constexpr int TILE = Cfg::kTile;
  constexpr int MT = D / 16;  // 16-wide blocks of head_dim
  constexpr int H = Cfg::kHalves;

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[NSTAGES];
  __shared__ __align__(8) uint64_t empty_bar[NSTAGES];

  const int part = blockIdx.x;
  const int kv_head = blockIdx.y;
  const int seq = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rows_log2 = p.rows_log2;
  const int rows = 1 << rows_log2;
  const int hstride = rows << 7;            // bytes between column blocks of one page
  const int page_bytes = 2 * H * hstride;   // K + V of one page

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], WARPS);
    }
    mbar_init_fence();
  }
  if (warp == WARPS && lane == 0) {
    tma_prefetch_desc(&k_map);
    if (!p.kv_fused) tma_prefetch_desc(&v_map);
  }
  __syncthreads();

  // Inputs written by the previous kernel in the stream are visible after this.
  pdl_wait_primary();

  const int seq_len = p.seq_lens[seq];
  const int pstart = part * p.partition_size;
  if (pstart >= seq_len) {
    // Empty sequence (single pass writes zeros) or a partition past the end
    // (skipped; the merge kernel reads only live partitions).
    if (!p.split) write_zero_output<T, D>(p, seq, kv_head, threadIdx.x, Cfg::kThreads);
    pdl_launch_dependents();
    return;
  }
  const int pend = min(pstart + p.partition_size, seq_len);
  const int ntiles = (pend - pstart + TILE - 1) / TILE;

  if (warp == WARPS) {
    // ------------------------------------------------------------------ producer
    const int bs_log2 = p.bs_log2;
    const int lb0 = pstart >> bs_log2;
    const int nlb = ((pend - 1) >> bs_log2) - lb0 + 1;  // logical blocks this partition touches
    const int* bt = p.block_tables + static_cast<int64_t>(seq) * p.bt_stride + lb0;
    int cur = (lane < nlb) ? __ldg(bt + lane) : 0;
    int nxt = (32 + lane < nlb) ? __ldg(bt + 32 + lane) : 0;
    int base = 0;
    const uint64_t policy = l2_evict_first_policy();

    for (int t = 0; t < ntiles; ++t) {
      const int s = t % NSTAGES;
      if (!mbar_wait(&empty_bar[s], ((t / NSTAGES) & 1) ^ 1)) break;
      const int tstart = pstart + t * TILE;
      const int nops = (min(TILE, pend - tstart) + rows - 1) >> rows_log2;

      int pbs[TILE / 8];
      int offs[TILE / 8];
#pragma unroll
      for (int j = 0; j < TILE / 8; ++j) {
        int pb = 0, off = 0;
        if (j < nops) {
          const int tok = tstart + (j << rows_log2);
          const int rel = (tok >> bs_log2) - lb0;
          off = tok & ((1 << bs_log2) - 1);
          while (rel >= base + 32) {  // warp-uniform
            base += 32;
            cur = nxt;
            nxt = (base + 32 + lane < nlb) ? __ldg(bt + base + 32 + lane) : 0;
          }
          pb = __shfl_sync(0xffffffffu, cur, rel - base);
        }
        pbs[j] = pb;
        offs[j] = off;
      }

      if (lane == 0) {
        uint8_t* dst = smem + s * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(nops * page_bytes));
#pragma unroll
        for (int j = 0; j < TILE / 8; ++j) {
          if (j < nops) {
            uint8_t* page = dst + j * page_bytes;
            tma_load_5d(page, &k_map, 0, offs[j], 0, kv_head, pbs[j], &full_bar[s], policy);
            if (!p.kv_fused) tma_load_5d(page + H * hstride, &v_map, 0, offs[j], 0, kv_head, pbs[j], &full_bar[s], policy);
          }
        }
      }
      __syncwarp();
    }
    pdl_launch_dependents();
    // The producer then helps with the merge (it holds no partial state).
    named_bar_sync(1, Cfg::kThreads);
    named_bar_sync(1, Cfg::kThreads);
    float* red = reinterpret_cast<float*>(smem);
    write_partition_result<T, D, WARPS>(p, red, seq, kv_head, part, seq_len, threadIdx.x, Cfg::kThreads,
                                        [] { named_bar_sync(1, Cfg::kThreads); });
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

  // Per-lane shared-memory offsets (bytes from a stage base) of the rows this
  // lane addresses in ldmatrix, and their swizzle phases.
  const int r0 = warp * kSubTokens;  // first tile row of this warp
  const int k_row = r0 + (lane & 7) + (((lane >> 3) & 1) << 3);  // K as A (row-major)
  const int k_chunk = lane >> 4;                                 // 0: k 0-7, 1: k 8-15
  const int v_row = r0 + (lane & 7) + ((lane >> 4) << 3);        // V^T as A (via .trans)
  const int v_chunk = (lane >> 3) & 1;                           // 0: d 0-7, 1: d 8-15
  const int k_off = (k_row >> rows_log2) * page_bytes + ((k_row & (rows - 1)) << 7);
  const int k_sw = k_row & 7;
  const int v_off = (v_row >> rows_log2) * page_bytes + H * hstride + ((v_row & (rows - 1)) << 7);
  const int v_sw = v_row & 7;

  const uint32_t smem_base = smem_u32(smem);
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % NSTAGES;
    const uint32_t parity = (t / NSTAGES) & 1;
    const int sub0 = pstart + t * TILE + r0;  // first token of this warp's 16
    if (sub0 < pend) {
      if (!mbar_wait(&full_bar[s], parity)) break;
      const uint32_t sb = smem_base + s * Cfg::kStageBytes;

      // S^T[16 tokens][8 heads] = K Q^T, two accumulator chains
      float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      float sc2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int kk = 0; kk < MT; ++kk) {
        const int chunk = ((kk & 3) << 1) + k_chunk;
        const uint32_t addr = sb + k_off + (kk >> 2) * hstride + ((chunk ^ k_sw) << 4);
        uint32_t a[4];
        ldmatrix_x4(a, addr);
        if (kk & 1)
          Mma<T>::run(sc2, a, qf[kk][0], qf[kk][1]);
        else
          Mma<T>::run(sa, a, qf[kk][0], qf[kk][1]);
      }
      float sc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[i] = (sa[i] + sc2[i]) * p.scale_log2;
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

      if (sub0 + kSubTokens > pend) {
        // Rows of tokens >= pend hold whatever the page (or an earlier tile)
        // left there; P is 0 for them but 0 * NaN is NaN, so clear them.
        const int first_bad = pend - (sub0 - r0);
        for (int i = lane; i < kSubTokens * H * 8; i += 32) {
          const int row = r0 + i / (H * 8);
          const int rem = i % (H * 8);
          if (row >= first_bad) {
            const int roff = (row >> rows_log2) * page_bytes + ((row & (rows - 1)) << 7);
            st_shared_zero16(sb + roff + (H + (rem >> 3)) * hstride + ((rem & 7) << 4));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int chunk = ((mt & 3) << 1) + v_chunk;
        const uint32_t addr = sb + v_off + (mt >> 2) * hstride + ((chunk ^ v_sw) << 4);
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
  // ring can be reused for the cross-warp merge once all warps are here.
  named_bar_sync(1, Cfg::kThreads);
  using Red = RedLayout<D>;
  constexpr int R = Red::kRow;
  float* red = reinterpret_cast<float*>(smem);
  float* red_o = Red::o(red);
  float* red_m = Red::m(red, WARPS);
  float* red_l = Red::l(red, WARPS);
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
  named_bar_sync(1, Cfg::kThreads);
  write_partition_result<T, D, WARPS>(p, red, seq, kv_head, part, seq_len, threadIdx.x, Cfg::kThreads,
                                      [] { named_bar_sync(1, Cfg::kThreads); });
}

}  // namespace dkb
