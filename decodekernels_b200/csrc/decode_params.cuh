// Parameters shared by the partition kernels and the merge kernel.
#pragma once

#include <limits.h>
#include <stdint.h>

namespace dkb {

constexpr int kTileTokens = 64;      // partition-size granularity; every pipeline tile divides it
constexpr int kSubTokens = 16;       // tokens per consumer warp per tile (mma M)
constexpr int kSimtThreads = 128;
constexpr int kMergeThreads = 256;
constexpr int kMaxGroup = 8;         // query heads per KV head (mma N)
constexpr int kMaxPeers = 8;         // GPUs of a peer-memory group (DK_MAX_PEERS)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Everything a launch needs besides the TMA descriptors.  Strides are in
// elements.  Field meanings follow DecodeKernels' PagedAttnParams
// (csrc/paged_attention.cuh:39-58) plus the planner's outputs.
struct DecodeParams {
  void* out;
  const void* q;
  const void* k_cache;  // read directly by the CUDA-core path only
  const void* v_cache;
  const int* block_tables;
  const int* seq_lens;
  float* tmp_out;
  float* max_logits;
  float* exp_sums;
  int* merge_counters;  // non-null: the last partition of each (seq, kv_head) merges (no merge kernel)
  int64_t q_stride_seq, q_stride_head;
  int64_t out_stride_seq, out_stride_head;
  int64_t k_stride_block, k_stride_token, k_stride_head;
  int64_t v_stride_block, v_stride_token, v_stride_head;
  int64_t bt_stride;
  int num_seqs;
  int num_q_heads;
  int num_kv_heads;
  int group;           // num_q_heads / num_kv_heads
  int max_seq_len;     // host-side bound on seq_lens; longer lengths count as this
  int block_size;
  int num_blocks;      // cache blocks; ids outside [0, num_blocks) read as zeros
  int bs_log2;         // log2(block_size) (TMA path: power-of-two block sizes)
  int rows_log2;       // log2 of token rows per TMA box: min(block_size, tile)
  int partition_size;  // tokens per partition, a multiple of kTileTokens
  int num_partitions;  // partitions in the grid
  int ws_partitions;   // workspace row stride (capacity)
  int split;           // 1: partitions write the workspace and the merge kernel writes out
  int kv_fused;        // 1: one tensor map covers K and V (vLLM's interleaved K|V rows)
  int lse_mode;        // 1: `out` is fp32 rows [o (head_dim) | lse | 3 pad] per (seq, q_head), not T
  float scale_log2;    // softmax scale * log2(e) (* k_scale for e4m3 caches)
  float v_scale;       // e4m3 caches: V = code * v_scale (1 otherwise), applied to the partition results
  int kv_fp8;          // 1: the caches hold e4m3 bytes
  int compact;         // 1: live work items numbered densely (compact_coords); CTA b runs items b, b + G, ...
  int persistent;      // 1 (with compact): the grid is one wave of resident CTAs
  // Partition size chosen on the device (fit_partition_size) when fit_slots > 0:
  // a multiple of fit_gran tokens in [fit_min_partition, partition_size].
  int fit_slots;          // resident CTAs of one wave of the partition kernel; 0: partition_size as planned
  int fit_min_partition;  // smallest size the workspace rows allow (num_partitions >= ceil(max_seq_len / it))
  int fit_gran;           // tokens: whole tiles of the partition kernel
  // (With a fitted size the workspace's last row of (sequence 0, query head
  // 0), which no partition reaches, carries the chosen size to the merge
  // kernel: fit_size_slot.)
  // Head all-gather fused into the output stores (dk_paged_attention_decode_gather):
  // with peer_world > 0 every output row goes, instead of to `out`, to slot
  // (call parity) of every rank's receive buffer [2][num_seqs, peer_q_heads, D]
  // at head peer_head0 + q_head; the parity is that of peer_state[0] + 1 (the
  // gathers completed so far + 1, read on the device).
  void* peer_recv[kMaxPeers];
  const uint32_t* peer_state;
  int64_t peer_slot_elems;  // num_seqs * peer_q_heads * D
  int peer_world;
  int peer_head0;
  int peer_q_heads;
};

// (partition, kv_head, seq) of this CTA in the 1-D grid, sequence-major:
// a (seq, kv_head)'s partitions are consecutive, so a long sequence's work is
// spread over the whole grid.  (Partition-major order, which pushes the
// early-exit CTAs past short sequences' ends to the back, measured 10% slower
// on skewed lengths -- it also pushes long sequences' last partitions into
// the tail -- and within 2% elsewhere.)
__device__ __forceinline__ void cta_coords(int num_partitions, int num_kv_heads, int& part, int& kv_head, int& seq) {
  const unsigned b = blockIdx.x;
  const unsigned np = static_cast<unsigned>(num_partitions);
  const unsigned pair = b / np;
  part = static_cast<int>(b - pair * np);
  seq = static_cast<int>(pair / static_cast<unsigned>(num_kv_heads));
  kv_head = static_cast<int>(pair - static_cast<unsigned>(seq) * static_cast<unsigned>(num_kv_heads));
}

// Compact grid: the live work items -- every (seq, kv_head, partition) with
// partition < max(1, ceil(L / partition_size)), L = min(seq_lens[seq],
// max_seq_len), in sequence-major order as above -- numbered densely; CTA b
// of a grid of G runs items b, b + G, ... (G is a few waves of resident
// CTAs, so it is usually one item).  For lengths far below max_seq_len most
// CTAs of the dense grid have no tokens, and interleaved with the live ones
// they slow the hardware's dispatch of the live CTAs (c4 with e4m3 caches:
// 938 live CTAs of 8192).  An empty sequence keeps its partition-0 item (it
// may write zeros).
constexpr int kCompactMaxSeqs = 512;
// The compact kernels are instantiated per lane capacity (sequences per
// lane of the warp that scans the lengths): 4 for up to 128 sequences, 16 for
// up to kCompactMaxSeqs.  The scans are unrolled over that capacity, and the
// small instance's shorter code measured faster at every CTA's start (c4
// 76.2 -> 75.3 us, c4f8 45.7 -> 44.2 us; the large one's prologue waited on
// instruction fetch).
constexpr int kCompactSmallPerLane = 4;
constexpr int kCompactPerLane = kCompactMaxSeqs / 32;
constexpr int compact_per_lane(int num_seqs) {
  return num_seqs <= 32 * kCompactSmallPerLane ? kCompactSmallPerLane : kCompactPerLane;
}

// Item `target` of the compact numbering, computed by one warp (all 32 lanes):
// lane l loads the lengths of sequences [l * per, (l + 1) * per) in one
// batch, a warp scan of the lanes' item counts finds the owner lane by
// ballot, and the owner walks its sequences.  Also returns the item's
// sequence length (clamped to [0, max_seq_len]).  False past the last item.
// `partition_size` is the size in force for this launch (p.partition_size, or
// fit_partition_size's choice).  STAGED: the lengths come from `staged`, the
// clamped copy fit_partition_size left in shared memory, else from
// p.seq_lens (one kind of load per instance, none issued speculatively).
// PER: the instance's lane capacity (num_seqs <= 32 * PER).
template <int PER, bool STAGED = false>
__device__ __forceinline__ bool compact_coords(const DecodeParams& p, const int* staged, unsigned target, int lane,
                                               int partition_size, int& part, int& kv_head, int& seq, int& seq_len) {
  const int per = (p.num_seqs + 31) >> 5;  // <= PER
  const int first = lane * per;
  const unsigned ps = static_cast<unsigned>(partition_size);
  const unsigned hkv = static_cast<unsigned>(p.num_kv_heads);
  int len[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j)
    len[j] = j < per && first + j < p.num_seqs
                 ? max(min(STAGED ? staged[first + j] : __ldg(p.seq_lens + first + j), p.max_seq_len), 0)
                 : -1;
  unsigned parts[PER];
  unsigned mine = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    parts[j] = 0;
    if (j >= per) continue;  // warp-uniform: no lane has a sequence here, and no division runs for it
    parts[j] = len[j] < 0 ? 0u : 1u;  // an empty sequence keeps one item
    if (len[j] > static_cast<int>(ps)) parts[j] = (static_cast<unsigned>(len[j]) + ps - 1) / ps;
    mine += parts[j];
  }
  mine *= hkv;
  unsigned incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (target >= __shfl_sync(0xffffffffu, incl, 31)) return false;
  const int owner = __ffs(__ballot_sync(0xffffffffu, incl > target)) - 1;
  int f_seq = 0, f_head = 0, f_part = 0, f_len = 0;
  if (lane == owner) {
    // walk to the item's sequence, then one division splits the remainder
    unsigned r = target - (incl - mine);
    bool found = false;
    unsigned f_parts = 1;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const unsigned items = parts[j] * hkv;
      if (!found && r < items) {
        found = true;
        f_seq = first + j;
        f_parts = parts[j];
        f_len = len[j];
      } else if (!found) {
        r -= items;
      }
    }
    f_head = static_cast<int>(r / f_parts);
    f_part = static_cast<int>(r - static_cast<unsigned>(f_head) * f_parts);
  }
  seq = __shfl_sync(0xffffffffu, f_seq, owner);
  kv_head = __shfl_sync(0xffffffffu, f_head, owner);
  part = __shfl_sync(0xffffffffu, f_part, owner);
  seq_len = __shfl_sync(0xffffffffu, f_len, owner);
  return true;
}

// Where the partition kernel leaves a fitted partition size for the merge
// kernel (as float bits): exp_sums' last row of (sequence 0, query head 0).
// The planner keeps that row out of every partition's reach.
__device__ __forceinline__ float* fit_size_slot(const DecodeParams& p) {
  return p.exp_sums + (p.ws_partitions - 1);
}

// Partition size fitted to the batch's lengths: the smallest multiple of
// p.fit_gran in [p.fit_min_partition, p.partition_size] whose live items
// (compact_coords' numbering) number at most p.fit_slots, so that every item
// starts in the first wave of resident CTAs and the kernel takes about as
// long as its longest partition; the planned p.partition_size when even its
// items do not fit (its waves were sized for lengths near max_seq_len).  The
// host sees only max_seq_len: a batch whose lengths sit far below it (a
// lognormal spread, for example) leaves most of a wave idle at the planned
// size.  FlashInfer's decode planner searches its KV chunk size for the same
// bound, from host-side lengths; here the lengths stay on the device, so a
// captured CUDA graph replays with the choice of each step's batch.
//
// All `nthreads` threads of the CTA call it (it holds __syncthreads).  The
// clamped lengths go to shared memory once (`lens`, num_seqs ints; held in
// registers instead, the read-only loads were re-issued for every candidate
// under the partition kernel's register pressure); the partition kernel's
// first compact_coords reads them from there too.  With t = ceil(L / gran)
// per sequence, T = sum t over the N sequences and c = fit_slots / num_kv_heads,
// the items at m tiles per partition, sum max(1, ceil(t / m)), lie in
// [T / m, T / m + N]: no m < T / c fits, and every m >= T / (c - N) does, so
// only sizes in [ceil(T / c), ceil(T / (c - N))] need counting, within the
// planned size (8 for e4m3 c4, against 39 in the workspace's range; none
// when ceil(T / c) is above the planned size, which then stays).  Warp w counts 4 of them at a
// time, (m0 + 4w .. m0 + 4w + 3) * gran, then the next 4 * warps: lane l sums
// max(1, ceil(t / m)) over sequences l, l + 32, ..., then one warp reduction
// per candidate (the four chains are independent); `best` (shared) keeps
// the smallest fitting candidate.  ceil(t / m) = umulhi(t + m - 1,
// ceil(2^32 / m)), exact for (t + m - 1) * (m - 1) < 2^32: the planner fits
// only max_seq_len <= 2^22, and sizes of 512..8192 tokens in tiles of 32 to
// 128 (a power of two), so t <= 2^17 and 4 <= m <= 2^8.  Every CTA of a
// launch computes the same value; CTA 0 leaves it in fit_size_slot for the
// merge kernel.
template <int PER>  // the instance's lane capacity (num_seqs <= 32 * PER)
__device__ __forceinline__ int fit_partition_size(const DecodeParams& p, int* lens, int* best, int tid, int nthreads) {
  constexpr int K = 4;  // candidates per warp and round
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int warps = nthreads >> 5;
  const int gran = p.fit_gran;
  const int gran_log2 = __ffs(gran) - 1;
  const int nj = (p.num_seqs + 31) >> 5;  // slots j holding a sequence in some lane (warp-uniform)
  if (tid == 0) *best = INT_MAX;
  for (int s = tid; s < p.num_seqs; s += nthreads) lens[s] = max(min(__ldg(p.seq_lens + s), p.max_seq_len), 0);
  __syncthreads();
  uint32_t tiles[PER];
  unsigned total = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    tiles[j] = 0;
    const int s = lane + 32 * j;
    if (j < nj && s < p.num_seqs) {
      tiles[j] = static_cast<uint32_t>((lens[s] + gran - 1) >> gran_log2);
      total += tiles[j];
    }
  }
  total = __reduce_add_sync(0xffffffffu, total);
  const unsigned cap = static_cast<unsigned>(p.fit_slots / p.num_kv_heads);  // items per KV head
  const unsigned nseq = static_cast<unsigned>(p.num_seqs);
  const int hi = p.partition_size / gran;
  const int lo = max(p.fit_min_partition / gran, cap > 0 ? static_cast<int>((total + cap - 1) / cap) : hi + 1);
  int top = hi;  // the largest size that still needs counting (none when lo > hi)
  if (cap > nseq) top = min(hi, max(lo, static_cast<int>((total + cap - nseq - 1) / (cap - nseq))));
#pragma unroll 1
  for (int m0 = lo + K * warp; m0 <= top; m0 += K * warps) {
    uint32_t magic[K];
    unsigned n[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      magic[k] = 0xffffffffu / static_cast<uint32_t>(min(m0 + k, top)) + 1u;  // ceil(2^32 / m), m >= 2
      n[k] = 0;
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if (j >= nj) break;
      if (lane + 32 * j < p.num_seqs) {
#pragma unroll
        for (int k = 0; k < K; ++k)
          n[k] += max(1u, __umulhi(tiles[j] + static_cast<uint32_t>(min(m0 + k, top) - 1), magic[k]));
      }
    }
#pragma unroll
    for (int k = 0; k < K; ++k) n[k] = __reduce_add_sync(0xffffffffu, n[k]);
    if (lane == 0) {
      int fit = INT_MAX;
#pragma unroll
      for (int k = K - 1; k >= 0; --k)  // the smallest of the four that fits
        if (m0 + k <= top && n[k] <= cap) fit = m0 + k;
      if (fit != INT_MAX) atomicMin(best, fit);
    }
  }
  __syncthreads();
  const int b = *best;
  return b == INT_MAX ? p.partition_size : b * gran;
}

}  // namespace dkb
