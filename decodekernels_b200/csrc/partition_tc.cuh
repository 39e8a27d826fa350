// Partition kernel for e4m3 KV caches on the 5th-generation tensor cores
// (tcgen05, kind::f8f6f4), head_dim 128.  Same work item, inputs and
// results as the TMA partition kernel (one CTA per (partition, kv_head, seq),
// all `group` query heads of the KV head), but no cache byte is ever
// converted: the tensor cores read the e4m3 K and V tiles straight from the
// TMA ring.
//
// * Warp 0 (producer): per page of a 128-token tile, one TMA box of K rows
//   into the stage's K region and one of V rows into its V region (row r of
//   the tile at r * 128 bytes, 128-byte swizzled), so both regions are the
//   canonical 128-byte-swizzle operand layouts: K as K-major A (token rows),
//   V as MN-major A of V^T (d contiguous).  Block ids are loaded one tile
//   ahead by the lane that issues the page, as in the TMA kernel.
// * Warp 1 (MMA): allocates 64 TMEM columns (S^T twice, O^T) and one thread
//   issues, per tile t,
//     S^T[128 tok][16] = K Q^T        (M 128, N 16, K 128: 4 + 4 MMAs)
//   then, for tile t - 1 (so a tile's QK overlaps the previous softmax),
//     O^T[128 d][16] += V^T P^T       (M 128, N 16, K 128 tokens: 4 + 4 MMAs)
//   Q and P are 16-bit values split into two e4m3 parts, x = hi + lo with
//   hi = e4m3(x), lo = e4m3(x - hi) (about 8 significant bits together), each
//   product running once per part; the query is scaled by an exact power of
//   two into the e4m3 range first.  Heads past the group are zero rows.
// * Warps 2-5 (softmax, 128 threads): thread i owns token row i of S^T and,
//   at the end, row d = i of O^T.  Per tile: read S^T from TMEM, mask tokens
//   past the end, the tile's per-head max (warp redux + shared memory), a
//   lazy running max (raised only when a tile's max exceeds it by more than
//   2^8, and then O^T in TMEM is rescaled after the previous PV completes),
//   p = exp2(s - m) <= 2^8, the exp-sums, and P^T hi / lo bytes into shared
//   memory (double-buffered) for the PV MMA.  Stale V rows past the end are
//   cleared (0 * NaN would poison the MMA).
// * Completion flows through mbarriers: TMA -> full; tcgen05.commit -> S
//   ready, PV done, stage empty; softmax -> S free, P ready.  Every wait is
//   bounded; a wait that gives up is counted (dk_device_wait_timeouts) and
//   the CTA winds down.
// * The epilogue hands O^T, the running max and the exp-sums to the same
//   write_partition_result as the other partition kernels (split-K rows,
//   single-launch merge, LSE partials, fused head gather).
#pragma once

#include <type_traits>

#include "decode_params.cuh"
#include "dk_ptx.cuh"
#include "partition_epilogue.cuh"
#include "tc_ptx.cuh"
#include "tile_math.cuh"

namespace dkb {

template <int D, int NSTAGES>
struct TcConfig {
  static_assert(D == 128, "the tcgen05 e4m3 kernel covers head_dim 128");
  static constexpr int kTile = 128;                  // tokens per stage (the M of S^T)
  static constexpr int kRegion = kTile * 128;        // K (or V) rows of one stage
  static constexpr int kStageBytes = 2 * kRegion;
  static constexpr int kThreads = 192;               // producer, MMA, 4 softmax warps
  static constexpr int kQ = NSTAGES * kStageBytes;   // Q^T hi, lo: [16 heads][128 bytes] each
  static constexpr int kP = kQ + 2 * 2048;           // P^T [2 buffers][hi, lo][16 heads][128 tokens]
  static constexpr int kRed = kP;                    // epilogue scratch, over P^T once the last PV is done
  static constexpr int kRedBytes = RedLayout<D>::floats(1) * 4;
  static_assert(kRedBytes <= 4 * 2048, "epilogue scratch fits the P^T buffers");
  static constexpr int kSmemBytes = kP + 4 * 2048 + 1024;  // + alignment slack (2 CTAs per SM)
  static constexpr int kTmemCols = 64;               // S^T x 2 (16 columns each), O^T (16)
  static constexpr float kLazy = 8.0f;               // log2 headroom of the lazy running max
  static_assert(kTile / 8 <= 16, "one producer lane per page (K) and one per page (V)");
};

// Byte offset of (row, col) in a [rows][128 B] 128-byte-swizzled block.
__device__ __forceinline__ uint32_t sw128(int row, int col) {
  return static_cast<uint32_t>(row * 128 + ((((col >> 4) ^ (row & 7)) << 4) | (col & 15)));
}

// hi and lo e4m3 parts of (a, b) through f16 (exact residual): low byte = a.
__device__ __forceinline__ void split_e4m3x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const uint32_t x = Conv<__half>::pack2(a, b);
  hi = f16x2_to_e4m3x2(x);
  lo = f16x2_to_e4m3x2(hsub2_u32(x, e4m3x2_to_f16x2(hi)));
}

template <typename T, int D, int NSTAGES>
__global__ void __launch_bounds__(192, 1)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap k_map, const __grid_constant__ CUtensorMap v_map,
                           const DecodeParams p) {
  using Cfg = TcConfig<D, NSTAGES>;
  constexpr int TILE = Cfg::kTile;
  constexpr uint32_t IDESC_QK = idesc_e4m3(128, 16, false);
  constexpr uint32_t IDESC_PV = idesc_e4m3(128, 16, true);

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[NSTAGES];
  __shared__ __align__(8) uint64_t empty_bar[NSTAGES];
  __shared__ __align__(8) uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], q_bar;
  __shared__ uint32_t s_tmem;
  __shared__ float s_max[2][4][kMaxGroup];
  __shared__ float s_lsum[4][kMaxGroup];
  __shared__ uint32_t s_qmax;

  int part, kv_head, seq;
  cta_coords(p.num_partitions, p.num_kv_heads, part, kv_head, seq);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&pv_done[b], 1);
    }
    mbar_init(&q_bar, 4);
    mbar_init_fence();
    s_qmax = 0u;
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&k_map);
    if (!p.kv_fused) tma_prefetch_desc(&v_map);
  }
  __syncthreads();

  pdl_wait_primary();
  const int seq_len = min(p.seq_lens[seq], p.max_seq_len);
  const int pstart = part * p.partition_size;
  if (pstart >= seq_len) {
    if (partition_writes_zeros(p, part, seq_len)) write_zero_output<T, D>(p, seq, kv_head, threadIdx.x, Cfg::kThreads);
    pdl_launch_dependents();
    return;
  }
  const int pend = min(pstart + p.partition_size, seq_len);
  const int ntiles = (pend - pstart + TILE - 1) / TILE;

  if (warp == 1) tmem_alloc(&s_tmem, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t ring = smem_u32(smem);
  const uint32_t q_hi = ring + Cfg::kQ, q_lo = q_hi + 2048;
  const uint32_t p_base = ring + Cfg::kP;  // buffer b: hi at b * 4096, lo at b * 4096 + 2048

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    const int rows_log2 = p.rows_log2;
    const int rows = 1 << rows_log2;
    const int bs_log2 = p.bs_log2;
    const int bs_mask = (1 << bs_log2) - 1;
    const int kslot = lane & 15;
    const bool v_lane = lane >= 16;
    const int* bt = p.block_tables + static_cast<int64_t>(seq) * p.bt_stride;
    const uint64_t policy = l2_evict_first_policy();
    int pb = 0, off = 0;
    {
      const int tok = pstart + (kslot << rows_log2);
      if (tok < p.max_seq_len) {
        pb = __ldg(bt + (tok >> bs_log2));
        off = tok & bs_mask;
      }
    }
    const CUtensorMap* vm = p.kv_fused ? &k_map : &v_map;
    const int vcol = p.kv_fused ? 1 : 0;  // V's 128-byte column block in the fused K|V map
    for (int t = 0; t < ntiles; ++t) {
      const int s = t % NSTAGES;
      if (!mbar_wait(&empty_bar[s], ((t / NSTAGES) & 1) ^ 1)) break;
      const int tstart = pstart + t * TILE;
      const int nops = (min(TILE, pend - tstart) + rows - 1) >> rows_log2;
      if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(nops * rows * 128 * 2));
      __syncwarp();
      if (kslot < nops) {
        uint8_t* dst = smem + s * Cfg::kStageBytes + (v_lane ? Cfg::kRegion : 0) + (kslot << rows_log2) * 128;
        if (v_lane)
          tma_load_5d(dst, vm, 0, off, vcol, kv_head, pb, &full_bar[s], policy);
        else
          tma_load_5d(dst, &k_map, 0, off, 0, kv_head, pb, &full_bar[s], policy);
      }
      const int tok = tstart + TILE + (kslot << rows_log2);
      if (tok < pend) {
        pb = __ldg(bt + (tok >> bs_log2));
        off = tok & bs_mask;
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t t_o = tmem + 32;
      bool ok = mbar_wait(&q_bar, 0);
      tc_fence_after();
      for (int t = 0; ok && t <= ntiles; ++t) {
        if (t < ntiles) {
          const int s = t % NSTAGES;
          ok = mbar_wait(&full_bar[s], (t / NSTAGES) & 1) && (t < 2 || mbar_wait(&s_free[t & 1], ((t >> 1) - 1) & 1));
          if (!ok) break;
          tc_fence_after();
          const uint32_t kb = ring + s * Cfg::kStageBytes;
          const uint32_t t_s = tmem + 16 * (t & 1);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_e4m3(t_s, smem_desc_sw128(kb + 32 * k, 16, 1024), smem_desc_sw128(q_hi + 32 * k, 16, 1024),
                      IDESC_QK, k > 0);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_e4m3(t_s, smem_desc_sw128(kb + 32 * k, 16, 1024), smem_desc_sw128(q_lo + 32 * k, 16, 1024),
                      IDESC_QK, true);
          umma_commit(&s_full[t & 1]);
        }
        if (t >= 1) {
          const int u = t - 1;
          const int s = u % NSTAGES;
          ok = mbar_wait(&p_full[u & 1], (u >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          const uint32_t vb = ring + s * Cfg::kStageBytes + Cfg::kRegion;
          const uint32_t ph = p_base + (u & 1) * 4096, pl = ph + 2048;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_e4m3(t_o, smem_desc_sw128(vb + 4096 * k, Cfg::kRegion, 1024), smem_desc_sw128(ph + 32 * k, 16, 1024),
                      IDESC_PV, u > 0 || k > 0);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_e4m3(t_o, smem_desc_sw128(vb + 4096 * k, Cfg::kRegion, 1024), smem_desc_sw128(pl + 32 * k, 16, 1024),
                      IDESC_PV, true);
          umma_commit(&pv_done[u & 1]);
          umma_commit(&empty_bar[s]);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- softmax
    const int ts = threadIdx.x - 64;       // 0..127
    const int qd = warp & 3;               // TMEM lane quadrant this warp may access
    const int row = qd * 32 + lane;        // token row of S^T, and d row of O^T
    const uint32_t lane_addr = static_cast<uint32_t>(qd * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + Cfg::kRed);
    auto sync128 = [] { named_bar_sync(2, 128); };

    // Q^T hi / lo rows (heads), scaled by 2^sq into the e4m3 range; rows of
    // heads past the group, and P^T rows 8..15 of both buffers, are zeros.
    float qv[16];
    const int qh = ts >> 3, qc = ts & 7;   // threads 0..63: head qh, 16 columns from 16 qc
    if (ts < 64) {
      float mx = 0.0f;
      const T* qrow = static_cast<const T*>(p.q) + static_cast<int64_t>(seq) * p.q_stride_seq +
                      static_cast<int64_t>(kv_head * p.group + qh) * p.q_stride_head + qc * 16;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        qv[j] = qh < p.group ? Conv<T>::to_f32(qrow[j]) : 0.0f;
        mx = fmaxf(mx, fabsf(qv[j]));
      }
      atomicMax(&s_qmax, __float_as_uint(mx));
    } else {
      const int i = ts - 64;  // 64 threads: 64 x 16 B of Q rows 8..15 (hi, lo) and 256 x 16 B of P rows 8..15
      st_shared_zero16(q_hi + 1024 + i * 16);
      st_shared_zero16(q_lo + 1024 + i * 16);
#pragma unroll
      for (int b = 0; b < 4; ++b) st_shared_zero16(p_base + b * 2048 + 1024 + i * 16);
    }
    sync128();
    const float qmax = __uint_as_float(s_qmax);
    const int e = static_cast<int>((__float_as_uint(qmax) >> 23) & 0xFF) - 127;
    const int sq = qmax > 0.0f ? min(max(7 - e, -100), 100) : 0;  // max |q| 2^sq in [128, 256)
    if (ts < 64) {
      const float up = __uint_as_float(static_cast<uint32_t>(127 + sq) << 23);
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float x0 = qv[4 * j] * up, x1 = qv[4 * j + 1] * up, x2 = qv[4 * j + 2] * up, x3 = qv[4 * j + 3] * up;
        const uint32_t h0 = f32x2_to_e4m3x2(x0, x1);
        const uint32_t h1 = f32x2_to_e4m3x2(x2, x3);
        const float2 d0 = e4m3x2_to_f32x2(h0);
        const float2 d1 = e4m3x2_to_f32x2(h1);
        const uint32_t l0 = f32x2_to_e4m3x2(x0 - d0.x, x1 - d0.y);
        const uint32_t l1 = f32x2_to_e4m3x2(x2 - d1.x, x3 - d1.y);
        hw[j] = h0 | (h1 << 16);
        lw[j] = l0 | (l1 << 16);
      }
      const uint32_t o = sw128(qh, qc * 16);
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(q_hi + o), "r"(hw[0]), "r"(hw[1]), "r"(hw[2]),
                   "r"(hw[3])
                   : "memory");
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(q_lo + o), "r"(lw[0]), "r"(lw[1]), "r"(lw[2]),
                   "r"(lw[3])
                   : "memory");
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&q_bar);
    const float sl2 = p.scale_log2 * __uint_as_float(static_cast<uint32_t>(127 - sq) << 23);

    float m_run[kMaxGroup], l_run[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
      m_run[h] = -INFINITY;
      l_run[h] = 0.0f;
    }
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int s = t % NSTAGES;
      ok = mbar_wait(&s_full[t & 1], (t >> 1) & 1);
      if (!ok) break;
      tc_fence_after();
      uint32_t r[8];
      tmem_ld8(tmem + lane_addr + 16 * (t & 1), r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[t & 1]);
      const int tstart = pstart + t * TILE;
      const bool valid = tstart + row < pend;
      float sv[kMaxGroup];
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) sv[h] = valid ? __uint_as_float(r[h]) * sl2 : -INFINITY;
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) {
        const float mx = warp_max_f32(sv[h]);
        if (lane == 0) s_max[t & 1][qd][h] = mx;
      }
      sync128();
      bool rescale = false;
      float alpha[kMaxGroup];
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) {
        const float tmax = fmaxf(fmaxf(s_max[t & 1][0][h], s_max[t & 1][1][h]),
                                 fmaxf(s_max[t & 1][2][h], s_max[t & 1][3][h]));
        const float mn = tmax > m_run[h] + Cfg::kLazy ? tmax : m_run[h];
        alpha[h] = fast_exp2(m_run[h] - mn);  // 0 while m_run is -inf
        rescale |= mn != m_run[h];
        m_run[h] = mn;
      }
      if (rescale) {
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) l_run[h] *= alpha[h];
        if (t > 0) {  // O^T holds tiles 0..t-1 once PV(t-1) is done
          ok = mbar_wait(&pv_done[(t - 1) & 1], ((t - 1) >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          uint32_t o[8];
          tmem_ld8(tmem + 32 + lane_addr, o);
#pragma unroll
          for (int h = 0; h < kMaxGroup; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
          tmem_st8(tmem + 32 + lane_addr, o);
          tc_fence_before();
        }
      }
      float pr[kMaxGroup];
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) {
        pr[h] = fast_exp2(sv[h] - m_run[h]);  // 0 for masked tokens
        l_run[h] += pr[h];
      }
      if (t >= 2) {  // P^T buffer t & 1 was last read by PV(t - 2)
        ok = mbar_wait(&pv_done[t & 1], ((t >> 1) - 1) & 1);
        if (!ok) break;
      }
      if (!valid) {  // stale bytes of this token's V row: clear them
        const uint32_t vrow = ring + s * Cfg::kStageBytes + Cfg::kRegion + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) st_shared_zero16(vrow + c * 16);
      }
      const uint32_t ph = p_base + (t & 1) * 4096, pl = ph + 2048;
#pragma unroll
      for (int h = 0; h < kMaxGroup; h += 2) {
        uint32_t hi, lo;
        split_e4m3x2(pr[h], pr[h + 1], hi, lo);
        const uint32_t o0 = sw128(h, row), o1 = sw128(h + 1, row);
        asm volatile("st.shared.u8 [%0], %1;" ::"r"(ph + o0), "r"(hi & 0xFFu) : "memory");
        asm volatile("st.shared.u8 [%0], %1;" ::"r"(ph + o1), "r"(hi >> 8) : "memory");
        asm volatile("st.shared.u8 [%0], %1;" ::"r"(pl + o0), "r"(lo & 0xFFu) : "memory");
        asm volatile("st.shared.u8 [%0], %1;" ::"r"(pl + o1), "r"(lo >> 8) : "memory");
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t & 1]);
    }
    // ------------------------------------------------------------ epilogue
    const int last = ntiles - 1;
    if (ok) ok = mbar_wait(&pv_done[last & 1], (last >> 1) & 1);
    tc_fence_after();
    uint32_t o[8];
    tmem_ld8(tmem + 32 + lane_addr, o);  // row d = `row` of O^T, one column per head
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
      float l = l_run[h];
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1) l += __shfl_xor_sync(0xffffffffu, l, sh);
      if (lane == 0) s_lsum[qd][h] = l;
    }
    using Red = RedLayout<D>;
    float* red_o = Red::o(red);
    float* red_m = Red::m(red, 1);
    float* red_l = Red::l(red, 1);
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h)
      if (h < p.group) red_o[h * Red::kRow + row] = __uint_as_float(o[h]);
    sync128();
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {  // m_run is the same in every thread
      if (ts == h && h < p.group) {
        red_m[h] = m_run[h];
        red_l[h] = s_lsum[0][h] + s_lsum[1][h] + s_lsum[2][h] + s_lsum[3][h];
      }
    }
    sync128();
    pdl_launch_dependents();
    write_partition_result<T, D, 1>(p, red, seq, kv_head, part, seq_len, ts, 128, sync128);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Cfg::kTmemCols);
  if (warp < 2) pdl_launch_dependents();
}

}  // namespace dkb
