// Partition kernel, sm_100a fast path: TMA-staged KV pages + tensor-core math.
//
// One CTA per (partition, kv_head, seq) work item computes all `group` query
// heads of its KV head, so every K/V byte is read from HBM once
// (DecodeKernels' GQA-aware block, csrc/paged_attention.cuh:73-225,
// re-designed):
//
// * Warp WARPS (producer): lane k addresses page k of every tile -- it loads
//   that page's block id itself, one tile ahead -- and issues ONE 5-D TMA box
//   per page for K (lanes PAGES.. for V) -- or a single box for both when the
//   cache is vLLM's interleaved K|V buffer -- into an NSTAGES-deep
//   shared-memory ring.  The tensor maps are (128 bytes of columns, token,
//   column block, head, block) with the caches' real strides, so the vLLM and
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

#include <type_traits>

#include "decode_params.cuh"
#include "dk_ptx.cuh"
#include "partition_epilogue.cuh"
#include "tile_math.cuh"
#include "tile_math_fp8.cuh"

namespace dkb {

// WARPS consumer warps of 16 tokens each make a tile of 16 * WARPS tokens
// (64 for head_dim <= 128, 32 for head_dim 256 so that several CTAs fit on
// an SM); a tile divides the 64-token partition granularity.  KV_BYTES is the
// cache element size (2, or 1 for e4m3 caches).
template <int D, int NSTAGES, int WARPS, int KV_BYTES = 2, int SLICES = 1>
struct TmaConfig {
  static constexpr int kWarps = WARPS;
  static constexpr int kTile = kSubTokens * WARPS * SLICES;        // tokens per pipeline stage
  static constexpr int kThreads = (WARPS + 1) * 32;                // + one TMA producer warp
  static constexpr int kHalves = D * KV_BYTES / 128;               // 128-byte column blocks per row
  static constexpr int kTileBytes = kHalves * kTile * 128;         // K (or V) of one tile
  static constexpr int kStageBytes = 2 * kTileBytes;               // K + V
  static constexpr int kSmemBytes = NSTAGES * kStageBytes + 1024;  // + alignment slack
  // a tile of 64 tokens or fewer divides the partition granularity; larger
  // ones rely on the planner's partitions being whole tiles (the kernel masks
  // the rest of a partial tile either way)
  static_assert(kTileTokens % kTile == 0 || kTile % kTileTokens == 0, "tile and partition granularity");
  static_assert(kTile / 8 <= 16, "a tile spans at most 16 pages (two producer lanes each)");
  static_assert(RedLayout<D>::floats(WARPS) * 4 <= NSTAGES * kStageBytes, "merge scratch must fit");
};

// Stage layout: page-major.  Page j of a tile (rows = min(block_size, tile)
// token rows) occupies kPage = 2 * kHalves * rows * 128 bytes: the K column
// blocks [h][row][128 B] followed by the V column blocks.
//
// FP8: the caches hold e4m3 bytes (rows of D bytes, D / 128 column blocks);
// the consumers convert in registers (tile_math_fp8.cuh).  SLICES: 16-token
// slices per consumer warp and tile (2: the warp's two slices share one
// softmax update, for the e4m3 path at head_dim 128 whose consumers bound the
// throughput; the e4m3 path at 256 takes 1, for a ring small enough that
// registers, not shared memory, bound the CTAs per SM).
// MIN_CTAS: resident CTAs per SM the register allocation must allow (0: no
// constraint, the compiler's own choice).  COMPACT > 0: the grid is compact
// (compact_coords; COMPACT is the lane capacity of its length scans,
// kCompactSmallPerLane or kCompactPerLane) and a CTA runs items b, b + G, ...,
// carrying its ring position and barrier phases from item to item; 0: one CTA
// per (partition, kv_head, seq) of the dense grid (cta_coords).
template <typename T, int D, int NSTAGES, int WARPS, bool FP8 = false, int SLICES = 1, int MIN_CTAS = 0,
          int COMPACT = 0>
__global__ void __launch_bounds__((WARPS + 1) * 32, MIN_CTAS)
    paged_decode_tma_kernel(const __grid_constant__ CUtensorMap k_map, const __grid_constant__ CUtensorMap v_map,
                            const DecodeParams p) {
  using Cfg = TmaConfig<D, NSTAGES, WARPS, FP8 ? 1 : 2, SLICES>;
  constexpr int TILE = Cfg::kTile;
  constexpr int H = Cfg::kHalves;

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[NSTAGES];
  __shared__ __align__(8) uint64_t empty_bar[NSTAGES];
  __shared__ int s_item[4];  // compact grid: seq (-1: no item), kv_head, partition, length
  __shared__ int s_fit;      // compact grid: fit_partition_size's smallest fitting candidate
  __shared__ int s_ps;       // compact grid: the partition size in force
  __shared__ int s_abort;    // compact grid: a bounded wait gave up, so run no further item

  int part = 0, kv_head = 0, seq = 0;
  if constexpr (COMPACT == 0) cta_coords(p.num_partitions, p.num_kv_heads, part, kv_head, seq);
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
    if constexpr (COMPACT != 0) s_abort = 0;
  }
  if (warp == WARPS && lane == 0) {
    tma_prefetch_desc(&k_map);
    if (!p.kv_fused) tma_prefetch_desc(&v_map);
  }
  __syncthreads();

  // Inputs written by the previous kernel in the stream are visible after this.
  pdl_wait_primary();

  // Producer lane k (k < PAGES, the most pages a tile spans) addresses page k
  // of each tile and issues its box; lanes PAGES..2*PAGES-1 issue the V boxes
  // of separate K/V caches.  The block ids of an item's first tile are fetched
  // together with the length (entries below max_seq_len are inside the
  // block-table row), later ones one tile ahead.
  constexpr int PAGES = TILE / 8;  // block size >= 8 on this path
  const int kslot = lane % PAGES;
  const bool v_lane = lane >= PAGES && lane < 2 * PAGES && !p.kv_fused;
  const bool box_lane = warp == WARPS && (lane < PAGES || v_lane);
  const int bs_log2 = p.bs_log2;
  const int bs_mask = (1 << bs_log2) - 1;
  // The partition size in force: p.partition_size, or on the compact grid
  // fit_partition_size's choice when p.fit_slots > 0.  Read where it is used
  // (per item, not in the tile loop) so that it holds no register across it.
  auto part_size = [&]() -> int {
    if constexpr (COMPACT != 0)
      return *static_cast<volatile int*>(&s_ps);
    else
      return p.partition_size;
  };
  float* red = reinterpret_cast<float*>(smem);  // merge scratch, over the ring once an item's tiles are read

  // The tiles of one item (pstart < seq_len) and its result; g0 = tiles this
  // CTA ran before it (ring position and barrier phases).
  auto run_item = [&](int part, int kv_head, int seq, int seq_len, int pb, int off, uint32_t g0) {
    const int pstart = part * part_size();
    const int pend = min(pstart + part_size(), seq_len);
    const int ntiles = (pend - pstart + TILE - 1) / TILE;
    if (warp == WARPS) {
      // ------------------------------------------------------------------ producer
      const int* bt = p.block_tables + static_cast<int64_t>(seq) * p.bt_stride;
      const uint64_t policy = l2_evict_first_policy();
      for (int t = 0; t < ntiles; ++t) {
        const uint32_t u = g0 + t;
        const int s = static_cast<int>(u % NSTAGES);
        if (!mbar_wait(&empty_bar[s], ((u / NSTAGES) & 1) ^ 1)) {
          if constexpr (COMPACT != 0) s_abort = 1;
          break;
        }
        const int tstart = pstart + t * TILE;
        const int nops = (min(TILE, pend - tstart) + rows - 1) >> rows_log2;
        if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(nops * page_bytes));
        __syncwarp();  // the expected bytes are posted before any box can land
        if (box_lane && kslot < nops) {
          uint8_t* page = smem + s * Cfg::kStageBytes + kslot * page_bytes;
          if (v_lane)
            tma_load_5d(page + H * hstride, &v_map, 0, off, 0, kv_head, pb, &full_bar[s], policy);
          else
            tma_load_5d(page, &k_map, 0, off, 0, kv_head, pb, &full_bar[s], policy);
        }
        const int tok = tstart + TILE + (kslot << rows_log2);
        if (box_lane && tok < pend) {
          pb = __ldg(bt + (tok >> bs_log2));
          off = tok & bs_mask;
        }
      }
      pdl_launch_dependents();
      // The producer then helps with the merge (it holds no partial state).
      named_bar_sync(1, Cfg::kThreads);
      named_bar_sync(1, Cfg::kThreads);
      write_partition_result<T, D, WARPS>(p, red, seq, kv_head, part, seq_len, part_size(), threadIdx.x,
                                          Cfg::kThreads, [] { named_bar_sync(1, Cfg::kThreads); });
      return;
    }
    // -------------------------------------------------------------------- consumers
    using Tile = std::conditional_t<FP8, WarpAttentionFp8<T, D>, WarpAttention<T, D>>;
    Tile wa;
    wa.load_q_global(p, seq, kv_head, lane);
    wa.reset();
    float scale_log2 = p.scale_log2;
    if constexpr (FP8) scale_log2 *= wa.q_scale;
    const StageGeom<H> geom(rows_log2);
    const int r0 = warp * kSubTokens * SLICES;  // first tile row of this warp
    const uint32_t smem_base = smem_u32(smem);
    for (int t = 0; t < ntiles; ++t) {
      const uint32_t u = g0 + t;
      const int s = static_cast<int>(u % NSTAGES);
      const int sub0 = pstart + t * TILE + r0;  // first token of this warp's rows
      // Only the last tile can start past this warp's rows.  Such a warp must
      // not arrive on that stage's empty barrier here: with no full-barrier
      // wait to hold it back, its arrival could count towards the pending
      // phase of the tile NSTAGES earlier while a slower warp still reads that
      // tile, and the producer would overwrite it.  (A CTA that runs another
      // item arrives after this one, below.)
      if (sub0 >= pend) break;
      if (!mbar_wait(&full_bar[s], (u / NSTAGES) & 1)) {
        if constexpr (COMPACT != 0) s_abort = 1;
        break;
      }
      if constexpr (SLICES == 2)
        wa.slice2(smem_base + s * Cfg::kStageBytes, geom, r0, sub0, pend, scale_log2, lane);
      else
        wa.slice(smem_base + s * Cfg::kStageBytes, geom, r0, sub0, pend, scale_log2, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
    }
    pdl_launch_dependents();
    // Every tile's TMA writes have landed (warp 0 waits on every tile), so the
    // ring can be reused for the cross-warp merge once all warps are here.
    named_bar_sync(1, Cfg::kThreads);
    wa.to_red(red, WARPS, warp, p.group, lane);
    named_bar_sync(1, Cfg::kThreads);
    write_partition_result<T, D, WARPS>(p, red, seq, kv_head, part, seq_len, part_size(), threadIdx.x,
                                        Cfg::kThreads, [] { named_bar_sync(1, Cfg::kThreads); });
    if constexpr (COMPACT != 0) {
      // A warp with no rows in the last tile arrives on its empty barrier now,
      // when every warp has finished reading the ring (the epilogue's
      // barriers), so that the stage's phase completes before the next item.
      if (lane == 0 && pstart + (ntiles - 1) * TILE + r0 >= pend)
        mbar_arrive(&empty_bar[(g0 + ntiles - 1) % NSTAGES]);
    }
  };

  // The block ids of an item's first tile (producer lanes).
  auto first_page = [&](int part, int seq, int& pb, int& off) {
    const int tok = part * part_size() + (kslot << rows_log2);
    if (box_lane && tok < p.max_seq_len) {
      pb = __ldg(p.block_tables + static_cast<int64_t>(seq) * p.bt_stride + (tok >> bs_log2));
      off = tok & bs_mask;
    }
  };

  if constexpr (COMPACT == 0) {
    int pb = 0, off = 0;  // this lane's page of the next tile: block id and first row in the block
    first_page(part, seq, pb, off);
    const int seq_len = min(p.seq_lens[seq], p.max_seq_len);  // lengths above max_seq_len count as max_seq_len
    if (part * p.partition_size >= seq_len) {
      // Empty sequence (single pass writes zeros) or a partition past the end
      // (skipped; the merge kernel reads only live partitions).
      if (partition_writes_zeros(p, part, seq_len)) write_zero_output<T, D>(p, seq, kv_head, threadIdx.x, Cfg::kThreads);
      pdl_launch_dependents();
      return;
    }
    run_item(part, kv_head, seq, seq_len, pb, off, 0u);
  } else {
    // With a fitted size (e4m3 caches only: the 16-bit instances carry no
    // fit code) the first item's coordinates read the lengths that
    // fit_partition_size staged at the start of the ring (inputs of this
    // call, readable after the grid-dependency wait above).
    bool from_ring = false;
    if (FP8 && p.fit_slots > 0) {
      const int ps = fit_partition_size<COMPACT>(p, reinterpret_cast<int*>(smem), &s_fit, threadIdx.x, Cfg::kThreads);
      from_ring = true;
      if (threadIdx.x == 0) {
        s_ps = ps;
        if (blockIdx.x == 0 && p.split) *fit_size_slot(p) = __int_as_float(ps);  // for the merge kernel
      }
    } else if (threadIdx.x == 0) {
      s_ps = p.partition_size;
    }
    __syncthreads();
    uint32_t g0 = 0;
    for (unsigned item = blockIdx.x;; item += gridDim.x) {
      if (warp == 0) {
        int len = 0;
        bool live;
        if constexpr (FP8) {
          const int* staged = reinterpret_cast<const int*>(smem);
          live = from_ring ? compact_coords<COMPACT, true>(p, staged, item, lane, part_size(), part, kv_head, seq, len)
                           : compact_coords<COMPACT>(p, nullptr, item, lane, part_size(), part, kv_head, seq, len);
        } else {
          live = compact_coords<COMPACT>(p, nullptr, item, lane, part_size(), part, kv_head, seq, len);
        }
        if (from_ring) {
          // the ring's first TMA writes follow: order these reads of it before them
          fence_proxy_async_smem();
          from_ring = false;
        }
        if (lane == 0) {
          s_item[0] = live ? seq : -1;
          s_item[1] = kv_head;
          s_item[2] = part;
          s_item[3] = len;
        }
      }
      __syncthreads();
      seq = s_item[0];
      if (seq < 0) break;  // past the last item
      kv_head = s_item[1];
      part = s_item[2];
      const int seq_len = s_item[3];
      const int pstart = part * part_size();
      if (pstart >= seq_len) {
        // an empty sequence's item
        if (partition_writes_zeros(p, part, seq_len)) write_zero_output<T, D>(p, seq, kv_head, threadIdx.x, Cfg::kThreads);
      } else {
        int pb = 0, off = 0;
        first_page(part, seq, pb, off);
        run_item(part, kv_head, seq, seq_len, pb, off, g0);
        g0 += (min(pstart + part_size(), seq_len) - pstart + TILE - 1) / TILE;
      }
      // The next item's TMA writes reuse the ring that the merge scratch
      // occupied: order those generic accesses before them, and keep s_item
      // until every thread has read it.
      fence_proxy_async_smem();
      __syncthreads();
      if (s_abort) break;
    }
    pdl_launch_dependents();
  }
}

}  // namespace dkb
