// libdk_b200: paged-attention decode for B200 (sm_100a) behind a C ABI
// (include/dk_paged_attention.h).
//
// Host side of the library: argument validation (the checks DecodeKernels
// makes in csrc/ops.cu:48-106 and csrc/paged_attention.cuh:315-322), the
// per-shape planner (partition size, grid, path), TMA descriptor
// construction, and the launches (partition kernel, then the merge kernel
// when the plan splits), both with programmatic dependent launch so their
// prologues overlap the previous kernel's tail.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/dk_paged_attention.h"
#include "decode_params.cuh"
#include "merge_partitions.cuh"
#include "partition_simt.cuh"
#include "partition_tma.cuh"
#include "peer_exchange.cuh"
#include "reshape_and_cache.cuh"

namespace dkb {
namespace {

// 0.8.0: DkPlan.fit_min_partition (partition size fitted on the device); 0.7.0: dk_gather_heads,
// DK_FLAG_PERSISTENT; 0.6.0: dk_exchange_merge_lse; 0.5.0: e4m3 caches (DkPagedAttnArgs.kv_fp8 / k_scale /
// v_scale); 0.4.0: dk_paged_attention_decode_lse / dk_merge_lse; 0.3.0: dk_reshape_and_cache; 0.2.0:
// DkPagedAttnArgs.merge_counters
constexpr int kVersion = 800;
// Planner: partitions are sized so that the grid is about one wave of
// kPlanCtasPerSm CTAs per SM if every sequence had max_seq_len tokens, within
// at least kMinPartition tokens (overridable for tuning sweeps).
#ifndef DK_PLAN_CTAS_PER_SM
#define DK_PLAN_CTAS_PER_SM 2
#endif
#ifndef DK_PLAN_MIN_PARTITION
#define DK_PLAN_MIN_PARTITION 128
#endif
constexpr int kPlanCtasPerSm = DK_PLAN_CTAS_PER_SM;
constexpr int kMinPartition = DK_PLAN_MIN_PARTITION;

thread_local char g_last_error[512] = {0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int fail_cuda(cudaError_t e, const char* what) {
  return fail(static_cast<int>(e), "%s: %s", what, cudaGetErrorString(e));
}

constexpr int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }
constexpr int round_up(long long a, long long b) { return static_cast<int>(((a + b - 1) / b) * b); }

// Pipeline depth and consumer warps per head_dim (overridable at build time
// for tuning sweeps).  Two stages with several CTAs per SM beat deeper rings
// with fewer CTAs: the stream of each CTA has a serial per-tile cost, so
// bandwidth comes from concurrent CTAs.
#ifndef DK_TMA_STAGES_D64
#define DK_TMA_STAGES_D64 2
#endif
#ifndef DK_TMA_STAGES_D128
#define DK_TMA_STAGES_D128 2
#endif
#ifndef DK_TMA_STAGES_D256
#define DK_TMA_STAGES_D256 2
#endif
#ifndef DK_TMA_WARPS_D64
#define DK_TMA_WARPS_D64 4
#endif
#ifndef DK_TMA_WARPS_D128
#define DK_TMA_WARPS_D128 4
#endif
#ifndef DK_TMA_WARPS_D256
#define DK_TMA_WARPS_D256 2
#endif

// Resident CTAs per SM the head_dim-64 instances' registers must allow: six
// fit its 33 KB ring, and without the bound the compact instance spilled
// (72 registers, 8 bytes); with it both use 64 registers and spill nothing.
#ifndef DK_TMA_MIN_CTAS_D64
#define DK_TMA_MIN_CTAS_D64 6
#endif
template <int D>
struct TmaShape {
  static constexpr int kStages = D == 64 ? DK_TMA_STAGES_D64 : (D == 128 ? DK_TMA_STAGES_D128 : DK_TMA_STAGES_D256);
  static constexpr int kWarps = D == 64 ? DK_TMA_WARPS_D64 : (D == 128 ? DK_TMA_WARPS_D128 : DK_TMA_WARPS_D256);
  static constexpr int kSlices = 1;
  static constexpr int kMinCtas = D == 64 ? DK_TMA_MIN_CTAS_D64 : 0;
  using Cfg = TmaConfig<D, kStages, kWarps>;
};

template <int D>
constexpr int tma_stages() {
  return TmaShape<D>::kStages;
}

// e4m3 caches: at head_dim 128 each consumer warp takes two 16-token slices
// per tile (their math is the limit, not HBM), so a tile holds as many bytes
// as a 16-bit one.  At head_dim 256 one slice: a 33 KB ring instead of 65 KB
// lets registers, not shared memory, bound the CTAs per SM (4 instead of 3),
// and a fitted partition size then fills the larger wave (c4f8 49.3 -> 47.8
// us in back-to-back timing).
#ifndef DK_TMA_FP8_STAGES
#define DK_TMA_FP8_STAGES 2
#endif
#ifndef DK_TMA_FP8_SLICES_D128
#define DK_TMA_FP8_SLICES_D128 2
#endif
#ifndef DK_TMA_FP8_SLICES_D256
#define DK_TMA_FP8_SLICES_D256 1
#endif
#ifndef DK_TMA_FP8_WARPS_D128
#define DK_TMA_FP8_WARPS_D128 DK_TMA_WARPS_D128
#endif
#ifndef DK_TMA_FP8_WARPS_D256
#define DK_TMA_FP8_WARPS_D256 DK_TMA_WARPS_D256
#endif
// e4m3 head_dim 128: three CTAs of its 65 KB ring fit an SM, and the bound
// lets the registers follow (117-120 each, no spill; without it ptxas chose
// 96 and the compact instance spilled).  c3f8 45.2 -> 44.0 us, c2f8 57.5 ->
// 57.0 us.
#ifndef DK_TMA_FP8_MIN_CTAS_D128
#define DK_TMA_FP8_MIN_CTAS_D128 3
#endif
#ifndef DK_TMA_FP8_MIN_CTAS_D256
#define DK_TMA_FP8_MIN_CTAS_D256 0
#endif
template <int D>
struct TmaShapeFp8 {
  static constexpr int kStages = DK_TMA_FP8_STAGES;
  static constexpr int kWarps = D == 128 ? DK_TMA_FP8_WARPS_D128 : DK_TMA_FP8_WARPS_D256;
  static constexpr int kSlices = D == 128 ? DK_TMA_FP8_SLICES_D128 : DK_TMA_FP8_SLICES_D256;
  static constexpr int kMinCtas = D == 128 ? DK_TMA_FP8_MIN_CTAS_D128 : DK_TMA_FP8_MIN_CTAS_D256;
  using Cfg = TmaConfig<D, kStages, kWarps, 1, kSlices>;
};

int tma_tile_fp8(int D) { return D == 128 ? TmaShapeFp8<128>::Cfg::kTile : TmaShapeFp8<256>::Cfg::kTile; }

int tma_tile(int D) {
  return D == 64 ? TmaShape<64>::Cfg::kTile : (D == 128 ? TmaShape<128>::Cfg::kTile : TmaShape<256>::Cfg::kTile);
}

int smem_for(int path, int D, bool fp8 = false) {
  if (path == DK_PATH_TMA_MMA && fp8) return D == 128 ? TmaShapeFp8<128>::Cfg::kSmemBytes
                                                      : TmaShapeFp8<256>::Cfg::kSmemBytes;
  if (path == DK_PATH_TMA_MMA) {
    switch (D) {
      case 64: return TmaShape<64>::Cfg::kSmemBytes;
      case 128: return TmaShape<128>::Cfg::kSmemBytes;
      default: return TmaShape<256>::Cfg::kSmemBytes;
    }
  }
  switch (D) {
    case 64: return SimtConfig<64>::kSmemBytes;
    case 128: return SimtConfig<128>::kSmemBytes;
    default: return SimtConfig<256>::kSmemBytes;
  }
}

// ---------------------------------------------------------------------------
// Per-device facts, cached
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
int g_num_sms[kMaxDevices] = {0};

int num_sms(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_num_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    g_num_sms[dev] = n;
  }
  return g_num_sms[dev];
}

// Opt every kernel that needs more than 48 KB of dynamic shared memory in,
// once per (kernel, device).
template <typename Kernel>
// Dynamic shared memory above 48 KB needs an opt-in, and the partition
// kernels want the whole carveout as shared memory (their KV traffic bypasses
// L1) so that as many CTAs as the ring allows stay resident.
cudaError_t ensure_smem_attr(Kernel kernel, int smem, int dev, bool* done) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (dev >= 0 && dev < kMaxDevices && done[dev]) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  if (smem > 48 * 1024) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) done[dev] = true;
  return e;
}

// ---------------------------------------------------------------------------
// Validation (DecodeKernels csrc/ops.cu:48-106, csrc/paged_attention.cuh:315-322)
// ---------------------------------------------------------------------------
bool aligned(const void* p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

int validate(const DkPagedAttnArgs* a) {
  if (a == nullptr) return fail(1, "dk_paged_attention_decode: args is NULL");
  if (a->dtype != DK_DTYPE_FLOAT16 && a->dtype != DK_DTYPE_BFLOAT16)
    return fail(1, "paged_attention_decode: expected float16 or bfloat16 (dtype code %d)", a->dtype);
  if (a->num_seqs < 0 || a->num_seqs > 65535) return fail(1, "num_seqs must be in [0, 65535]");
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256)
    return fail(1, "head_dim must be 64, 128 or 256, got %d", a->head_dim);
  if (a->num_kv_heads <= 0 || a->num_q_heads <= 0 || a->num_q_heads % a->num_kv_heads != 0)
    return fail(1, "num_q_heads must be a multiple of num_kv_heads");
  if (a->num_q_heads / a->num_kv_heads > DK_MAX_GQA_GROUP)
    return fail(1, "GQA group size above %d is not supported", DK_MAX_GQA_GROUP);
  if (a->block_size <= 0) return fail(1, "block_size must be positive");
  if (a->max_seq_len < 0) return fail(1, "max_seq_len must be non-negative");
  if (a->max_partitions < 0) return fail(1, "max_partitions must be non-negative");
  if (a->partition_size < 0 || a->partition_size % DK_TILE_TOKENS != 0)
    return fail(1, "partition_size must be 0 (planner) or a positive multiple of %d", DK_TILE_TOKENS);
  if (a->kv_fp8 != 0 && a->kv_fp8 != 1) return fail(1, "kv_fp8 must be 0 or 1");
  if (a->kv_fp8 && !(a->k_scale > 0.0f && a->v_scale > 0.0f && a->k_scale < INFINITY && a->v_scale < INFINITY))
    return fail(1, "fp8 KV cache: k_scale and v_scale must be positive and finite");
  if (a->num_seqs == 0) return 0;
  if (!a->out || !a->q || !a->k_cache || !a->v_cache || !a->block_tables || !a->seq_lens)
    return fail(1, "paged_attention_decode: NULL tensor pointer");
  if (a->num_blocks <= 0) return fail(1, "num_blocks must be positive");
  // Vectorised row loads: head_dim / 32 elements per lane (csrc/ops.cu:72-79).
  const int64_t vec = a->head_dim / 32;
  const int64_t strides[6] = {a->k_stride_block, a->k_stride_token, a->k_stride_head,
                              a->v_stride_block, a->v_stride_token, a->v_stride_head};
  for (int64_t s : strides) {
    if (s < 0 || s % vec != 0) return fail(1, "KV-cache strides must be multiples of head_dim / 32 for vectorised loads");
  }
  const size_t esz = a->kv_fp8 ? 1 : 2;
  if (!aligned(a->k_cache, static_cast<size_t>(vec) * esz) || !aligned(a->v_cache, static_cast<size_t>(vec) * esz))
    return fail(1, "KV-cache pointers must be aligned to head_dim / 32 elements");
  if (a->max_partitions > 0 && (!a->tmp_out || !a->max_logits || !a->exp_sums))
    return fail(1, "split-K workspace pointers are NULL but max_partitions > 0");
  if (a->max_partitions > 0 && (!aligned(a->tmp_out, 16) || !aligned(a->max_logits, 4) || !aligned(a->exp_sums, 4)))
    return fail(1, "split-K workspace: tmp_out must be 16-byte aligned, max_logits / exp_sums 4-byte aligned");
  if (a->merge_counters != nullptr && !aligned(a->merge_counters, 4))
    return fail(1, "merge_counters must be 4-byte aligned");
  return 0;
}

// ---------------------------------------------------------------------------
// Planner
// ---------------------------------------------------------------------------
// Tokens per partition before workspace constraints.  The host knows only
// max_seq_len, so:
// * one sequence (lengths cannot vary): spread its work over ~one wave of
//   kPlanCtasPerSm CTAs per SM;
// * several sequences with fewer (sequence, kv_head) pairs than ~4 waves of
//   CTAs: lengths may vary, so cap a partition at kVariedBytes of K+V (1024
//   tokens at head_dim 128, 512 at 256) for balance;
// * many pairs: partitions up to kMaxBytes of K+V (4096 tokens at 128).
// Caps are in bytes because a CTA streams a roughly fixed number of bytes
// per second whatever the head size.  Always a multiple of 64 tokens, at
// least kMinPartition.
#ifndef DK_PLAN_VARIED_BYTES
#define DK_PLAN_VARIED_BYTES (512 * 1024)
#endif
#ifndef DK_PLAN_MAX_BYTES
#define DK_PLAN_MAX_BYTES (2 * 1024 * 1024)
#endif
#ifndef DK_FUSED_MERGE_MAX_BYTES
#define DK_FUSED_MERGE_MAX_BYTES (64 * 1024)
#endif
// Compact grid (compact_coords): from this many partitions per sequence,
// for up to kCompactMaxSeqs sequences (a warp scans them all in every CTA);
// the grid is this many waves of resident CTAs at most.
#ifndef DK_COMPACT_MIN_PARTITIONS
#define DK_COMPACT_MIN_PARTITIONS 16
#endif
#ifndef DK_COMPACT_WAVES
#define DK_COMPACT_WAVES 4
#endif
constexpr int kCompactMinPartitions = DK_COMPACT_MIN_PARTITIONS;
constexpr int kCompactWaves = DK_COMPACT_WAVES;
constexpr long long kFusedMergeMaxBytes = DK_FUSED_MERGE_MAX_BYTES;
constexpr long long kVariedBytes = DK_PLAN_VARIED_BYTES;
#ifndef DK_PLAN_VARIED_WAVES
#define DK_PLAN_VARIED_WAVES 8
#endif
constexpr int kVariedWaves = DK_PLAN_VARIED_WAVES;
constexpr long long kMaxBytes = DK_PLAN_MAX_BYTES;
// Partition size fitted on the device (fit_partition_size), for e4m3
// caches in batches of 2..kCompactMaxSeqs sequences with at most one
// (sequence, KV head) pair per SM: the planner's size (waves sized as if
// every sequence had max_seq_len tokens) is only an upper bound, and the
// partition kernel picks the smallest size down to kFitMinPartition tokens
// -- the reference's fixed partition size, so a workspace sized as its
// wrapper sizes it allows nearly the full range -- whose live items fit one
// wave.  An e4m3 CTA's time follows its tokens (its consumers' math is the
// limit), so a wave left idle by lengths spread far below max_seq_len is
// lost time: e4m3 c4 (MQA, lognormal lengths) has 323 items for 444
// resident CTAs at the planned 1728 tokens, 55.0 us, and 429 items at the
// fitted 1216, 47.2 us with the size fixed.  A 16-bit CTA shares HBM with
// the others, and c4 ran 76.5 us at 1728 against 77.5 at 1216: no fit.
#ifndef DK_FIT_MIN_PARTITION
#define DK_FIT_MIN_PARTITION 512
#endif
constexpr int kFitMinPartition = DK_FIT_MIN_PARTITION;

bool fit_shape(int num_seqs, int num_kv_heads, int max_seq_len, int sms) {
  const long long pairs = static_cast<long long>(num_seqs) * std::max(num_kv_heads, 1);
  // (max_seq_len <= 2^22 keeps fit_partition_size's fp32 ceil-division exact)
  return num_seqs > 1 && num_seqs <= kCompactMaxSeqs && pairs <= sms && max_seq_len > kFitMinPartition &&
         max_seq_len <= (1 << 22);
}

int desired_partition_size(int num_seqs, int num_kv_heads, int head_dim, int max_seq_len, int sms, int kv_bytes = 2) {
  const long long pairs = std::max<long long>(1, static_cast<long long>(num_seqs) * std::max(num_kv_heads, 1));
  const long long slots = static_cast<long long>(kPlanCtasPerSm) * sms;
  const long long work = pairs * std::max(max_seq_len, 1);
  const long long token_bytes = 2LL * kv_bytes * head_dim;  // K + V
  int ps = round_up((work + slots - 1) / slots, DK_TILE_TOKENS);
  long long cap = kMaxBytes / token_bytes;
  // Varying lengths balance over many CTAs: with few (sequence, KV head)
  // pairs, about kVariedWaves waves of CTAs if every sequence had
  // max_seq_len tokens, within [kVariedBytes, kMaxBytes].  In 16-bit tokens
  // whatever the cache: an e4m3 CTA's time follows its tokens (its math is
  // the limit), and e4m3 c2 measured 6% faster at 1024 tokens than at 2048.
  // (8 waves, against the former fixed kVariedBytes cap: a rank's share of c5
  // at 2 / 4 / 8 GPUs 1188 -> 1153, 601 -> 589, 310 -> 303 us; of e4m3 c5 at
  // 2 / 8 GPUs 672 -> 620, 190 -> 178 us; c4 85.3 -> 83.4, e4m3 c4 68.3 ->
  // 62.4 us; c2 unchanged.  16 waves was slower on c4.)
  if (num_seqs > 1 && pairs < 4 * slots) {
    const long long want = work / (static_cast<long long>(kVariedWaves) * slots);
    cap = std::min(cap, std::max(kVariedBytes / (4LL * head_dim), std::min(kMaxBytes / (4LL * head_dim), want)));
  }
  cap = std::max<long long>(DK_TILE_TOKENS, cap / DK_TILE_TOKENS * DK_TILE_TOKENS);
  return static_cast<int>(std::min<long long>(std::max(ps, kMinPartition), cap));
}

// Path choice: the TMA path needs 16-byte aligned bases and strides (the
// tensor-map rules) and a power-of-two block size of at least 8 tokens (so a
// 64-token tile is whole pages, or a 64-row slice of one page, and the
// 128-byte swizzle spans 8 rows of a page).
bool tma_eligible(const DkPagedAttnArgs& a) {
  if (a.flags & DK_FLAG_FORCE_SIMT) return false;
  const int bs = a.block_size;
  if (bs < 8 || (bs & (bs - 1)) != 0) return false;
  if (a.kv_fp8 && a.head_dim < 128) return false;  // e4m3 rows shorter than a 128-byte swizzle row
  const int64_t esz = a.kv_fp8 ? 1 : 2;
  if (!aligned(a.k_cache, 16) || !aligned(a.v_cache, 16)) return false;
  const int64_t sizes[3] = {a.num_blocks, a.block_size, a.num_kv_heads};
  const int64_t ks[3] = {a.k_stride_block, a.k_stride_token, a.k_stride_head};
  const int64_t vs[3] = {a.v_stride_block, a.v_stride_token, a.v_stride_head};
  for (int i = 0; i < 3; ++i) {
    if (sizes[i] <= 1) continue;  // the coordinate is always 0; the stride is never used
    if ((ks[i] * esz) % 16 != 0 || (vs[i] * esz) % 16 != 0) return false;
    if (ks[i] * esz >= (int64_t(1) << 40) || vs[i] * esz >= (int64_t(1) << 40)) return false;
  }
  return true;
}

// K and V are the two halves of one row (vLLM's [blocks, heads, bs, 2*D]
// buffer viewed as two [blocks, bs, heads, D] tensors): one map covers both.
bool kv_fused(const DkPagedAttnArgs& a) {
  return static_cast<const char*>(a.v_cache) == static_cast<const char*>(a.k_cache) + a.head_dim * (a.kv_fp8 ? 1 : 2) &&
         a.k_stride_block == a.v_stride_block && a.k_stride_token == a.v_stride_token &&
         a.k_stride_head == a.v_stride_head;
}

int ilog2(int x) {
  int r = 0;
  while ((1 << (r + 1)) <= x) ++r;
  return r;
}

void make_plan(const DkPagedAttnArgs& a, int dev, DkPlan* pl) {
  std::memset(pl, 0, sizeof(*pl));
  if (a.num_seqs == 0) {
    pl->path = DK_PATH_NONE;
    return;
  }
  pl->path = tma_eligible(a) ? DK_PATH_TMA_MMA : DK_PATH_SIMT;
  const int L = a.max_seq_len;
  int ps, parts;
  int fit_parts = 0;  // partitions at the planned size when the device fits it
  if (L <= 0) {
    ps = DK_TILE_TOKENS;
    parts = 1;
  } else if (a.max_partitions <= 0) {
    ps = round_up(L, DK_TILE_TOKENS);  // no workspace: one pass over the whole sequence
    parts = 1;
  } else {
    // granularity of a chosen size: whole tiles of the kernel that runs
    const int gran = a.kv_fp8 && pl->path == DK_PATH_TMA_MMA ? tma_tile_fp8(a.head_dim) : DK_TILE_TOKENS;
    ps = a.partition_size > 0 ? a.partition_size
                              : round_up(desired_partition_size(a.num_seqs, a.num_kv_heads, a.head_dim, L,
                                                                num_sms(dev), a.kv_fp8 ? 1 : 2),
                                         gran);
    parts = ceil_div(L, ps);
    if (parts > a.max_partitions) {  // the caller's workspace caps the partition count
      ps = round_up(ceil_div(L, a.max_partitions), gran);
      parts = ceil_div(L, ps);
    }
    if (a.partition_size <= 0 && pl->path == DK_PATH_TMA_MMA && a.kv_fp8 && a.max_partitions >= 2 &&
        fit_shape(a.num_seqs, a.num_kv_heads, L, num_sms(dev))) {
      // ps becomes the upper bound of the device's choice.  The rows cover
      // the smallest size the workspace allows plus one: the last row of
      // (sequence 0, query head 0) passes the chosen size to the merge
      // kernel (fit_size_slot), and no partition reaches it.
      const int lo = std::max(round_up(kFitMinPartition, gran), round_up(ceil_div(L, a.max_partitions - 1), gran));
      if (lo < ps) {
        pl->fit_min_partition = lo;
        fit_parts = parts;
        parts = ceil_div(L, lo) + 1;
      }
    }
  }
  pl->partition_size = ps;
  pl->num_partitions = parts;
  pl->split = parts > 1 ? 1 : 0;
  pl->num_ctas = static_cast<int32_t>(std::min<long long>(INT_MAX, 1LL * parts * a.num_kv_heads * a.num_seqs));
  pl->stages = pl->path != DK_PATH_TMA_MMA ? 0
               : a.kv_fp8                 ? DK_TMA_FP8_STAGES
                                          : (a.head_dim == 64 ? tma_stages<64>()
                                                              : (a.head_dim == 128 ? tma_stages<128>() : tma_stages<256>()));
  pl->smem_bytes = smem_for(pl->path, a.head_dim, a.kv_fp8 != 0);
  // Merge counters turn the merge into the last partition's epilogue, which
  // saves the merge kernel's launch and latency but costs every partition a
  // release + atomic round trip and leaves each pair's merge to one CTA.
  // Measured worth it when each pair's rows are small (c1 13.3 -> 12.x us,
  // c2 105.7 -> 103-105, c5 and a rank's share of c5 at 2 / 4 / 8 GPUs
  // 0.2-0.4% faster); large merges are faster with the separate kernel
  // (c3 86 vs 90.5 us, c4 83 vs 90 us).
  // (A fitted size counts at its upper bound: the device never picks
  // more partitions than fit one wave.)
  const long long merge_bytes =
      1LL * (fit_parts > 0 ? fit_parts : parts) * (a.num_q_heads / a.num_kv_heads) * (a.head_dim + 2) * 4;
  const bool small = merge_bytes <= kFusedMergeMaxBytes;
  const bool fused = pl->split && a.merge_counters != nullptr && (small || (a.flags & DK_FLAG_FORCE_FUSED_MERGE));
  pl->launches = pl->split && !fused ? 2 : 1;
}

// ---------------------------------------------------------------------------
// TMA descriptors
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    } else {
      cudaGetLastError();
    }
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  int esz;
  int64_t strides[3];
  int64_t sizes[3];
  int rows;
  int col_blocks;
  int dev;
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};

struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};

constexpr int kMapCache = 32;
std::mutex g_map_mu;
MapEntry g_maps[kMapCache];
int g_map_next = 0;

// 5-D map over one cache view (or over K and V together when interleaved):
// dims (64 columns, token, 64-column block, head, block) with strides
// (2 B, token stride, 128 B, head stride, block stride).  The box is all
// `col_blocks` column blocks of `rows` token rows of one head of one page and
// lands in shared memory as [column block][row][128 B], 128-byte swizzled.
// esz: element size (2, or 1 for e4m3 bytes); a 128-byte column block holds
// 128 / esz elements.
int build_map(const void* ptr, int64_t s_block, int64_t s_tok, int64_t s_head, int64_t num_blocks, int block_size,
              int num_kv_heads, int col_blocks, int rows, int dev, CUtensorMap* out, int esz = 2) {
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  key.ptr = ptr;
  key.esz = esz;
  key.strides[0] = s_head;
  key.strides[1] = s_tok;
  key.strides[2] = s_block;
  key.sizes[0] = num_kv_heads;
  key.sizes[1] = block_size;
  key.sizes[2] = num_blocks;
  key.rows = rows;
  key.col_blocks = col_blocks;
  key.dev = dev;
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    for (auto& e : g_maps) {
      if (e.used && e.key == key) {
        *out = e.map;
        return 0;
      }
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(static_cast<int>(cudaErrorNotSupported), "cuTensorMapEncodeTiled is unavailable");
  // a dimension of size 1 is never stepped: any legal stride will do
  auto legal = [esz](int64_t size, int64_t stride_elems) -> cuuint64_t {
    const int64_t b = stride_elems * esz;
    return static_cast<cuuint64_t>(size <= 1 || b <= 0 || b % 16 != 0 ? 16 : b);
  };
  const cuuint32_t inner = static_cast<cuuint32_t>(128 / esz);
  const cuuint64_t gdim[5] = {inner, static_cast<cuuint64_t>(block_size), static_cast<cuuint64_t>(col_blocks),
                              static_cast<cuuint64_t>(num_kv_heads), static_cast<cuuint64_t>(num_blocks)};
  const cuuint64_t gstride[4] = {legal(block_size, s_tok), 128, legal(num_kv_heads, s_head),
                                 legal(num_blocks, s_block)};
  const cuuint32_t box[5] = {inner, static_cast<cuuint32_t>(rows), static_cast<cuuint32_t>(col_blocks), 1, 1};
  const cuuint32_t estride[5] = {1, 1, 1, 1, 1};
  CUtensorMap map;
  CUresult r = fn(&map, esz == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 5,
                  const_cast<void*>(ptr), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(1, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  *out = map;
  std::lock_guard<std::mutex> lk(g_map_mu);
  MapEntry& e = g_maps[g_map_next];
  g_map_next = (g_map_next + 1) % kMapCache;
  e.key = key;
  e.map = map;
  e.used = true;
  return 0;
}

// ---------------------------------------------------------------------------
// Launches
// ---------------------------------------------------------------------------
template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, int smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// K and V tensor maps (one map for both when K|V rows are interleaved).
template <int D>
int build_maps(const DkPagedAttnArgs& a, DecodeParams& p, int dev, CUtensorMap* kmap, CUtensorMap* vmap) {
  const int rows = 1 << p.rows_log2;
  p.kv_fused = kv_fused(a) ? 1 : 0;
  const int esz = a.kv_fp8 ? 1 : 2;
  const int cols = D * esz / 128;  // 128-byte column blocks of one K (or V) row
  if (int r = build_map(a.k_cache, a.k_stride_block, a.k_stride_token, a.k_stride_head, a.num_blocks, a.block_size,
                        a.num_kv_heads, (p.kv_fused ? 2 : 1) * cols, rows, dev, kmap, esz))
    return r;
  if (p.kv_fused) {
    *vmap = *kmap;  // unused
    return 0;
  }
  return build_map(a.v_cache, a.v_stride_block, a.v_stride_token, a.v_stride_head, a.num_blocks, a.block_size,
                   a.num_kv_heads, cols, rows, dev, vmap, esz);
}

// Resident CTAs per SM of the partition kernel a plan launches (0 when it
// cannot be queried, e.g. without a GPU).
template <typename Kernel>
int occupancy_of(Kernel kernel, int threads, int smem, int dev, bool* attr_done) {
  if (ensure_smem_attr(kernel, smem, dev, attr_done) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, static_cast<size_t>(smem)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

template <typename T, int D, int COMPACT>
int tma_occupancy(bool fp8, int dev) {
  if (fp8) {
    if constexpr (D >= 128) {
      using Shape = TmaShapeFp8<D>;
      static bool attr_done[kMaxDevices] = {false};
      return occupancy_of(
          paged_decode_tma_kernel<T, D, Shape::kStages, Shape::kWarps, true, Shape::kSlices, Shape::kMinCtas, COMPACT>,
          Shape::Cfg::kThreads, Shape::Cfg::kSmemBytes, dev, attr_done);
    }
    return 0;
  }
  using Shape = TmaShape<D>;
  static bool attr_done[kMaxDevices] = {false};
  return occupancy_of(
      paged_decode_tma_kernel<T, D, Shape::kStages, Shape::kWarps, false, Shape::kSlices, Shape::kMinCtas, COMPACT>,
      Shape::Cfg::kThreads, Shape::Cfg::kSmemBytes, dev, attr_done);
}

// Resident CTAs per SM of the partition kernel instance the plan runs (for a
// fitted partition size, the compact-grid instance whose one wave the device
// fills).
template <typename T, int D>
int partition_occupancy(const DkPlan& pl, bool fp8, int num_seqs, int dev) {
  if (pl.path == DK_PATH_TMA_MMA) {
    if (pl.fit_min_partition == 0) return tma_occupancy<T, D, 0>(fp8, dev);
    return compact_per_lane(num_seqs) == kCompactSmallPerLane ? tma_occupancy<T, D, kCompactSmallPerLane>(fp8, dev)
                                                              : tma_occupancy<T, D, kCompactPerLane>(fp8, dev);
  }
  static bool attr_done[kMaxDevices] = {false};
  return fp8 ? occupancy_of(paged_decode_simt_kernel<T, D, uint8_t>, kSimtThreads, SimtConfig<D>::kSmemBytes, dev,
                            attr_done)
             : occupancy_of(paged_decode_simt_kernel<T, D>, kSimtThreads, SimtConfig<D>::kSmemBytes, dev, attr_done);
}

int plan_occupancy(const DkPagedAttnArgs& a, const DkPlan& pl, int dev) {
  if (dev < 0 || pl.path == DK_PATH_NONE) return 0;
  const bool bf16 = a.dtype == DK_DTYPE_BFLOAT16;
  const bool fp8 = a.kv_fp8 != 0;
  switch (a.head_dim) {
    case 64:
      return bf16 ? partition_occupancy<__nv_bfloat16, 64>(pl, fp8, a.num_seqs, dev)
                  : partition_occupancy<__half, 64>(pl, fp8, a.num_seqs, dev);
    case 128:
      return bf16 ? partition_occupancy<__nv_bfloat16, 128>(pl, fp8, a.num_seqs, dev)
                  : partition_occupancy<__half, 128>(pl, fp8, a.num_seqs, dev);
    default:
      return bf16 ? partition_occupancy<__nv_bfloat16, 256>(pl, fp8, a.num_seqs, dev)
                  : partition_occupancy<__half, 256>(pl, fp8, a.num_seqs, dev);
  }
}

// CTAs of a compact grid (compact_coords): `waves` waves of the kernel's
// resident CTAs, at most one per work item of the dense grid.  The
// occupancy is queried once per kernel and device (cache; -1: unknown, which
// keeps the dense size).
template <typename Kernel>
unsigned compact_grid(Kernel kernel, int threads, int smem, int dev, int dense, int waves, int* cache) {
  if (dev < 0 || dev >= kMaxDevices) return static_cast<unsigned>(dense);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, static_cast<size_t>(smem)) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    cache[dev] = n > 0 ? n : -1;
  }
  if (cache[dev] < 0) return static_cast<unsigned>(dense);
  return static_cast<unsigned>(std::min<long long>(dense, 1LL * waves * cache[dev] * num_sms(dev)));
}

// One TMA partition kernel instance: e4m3 or 16-bit caches, dense grid
// (COMPACT 0) or compact grid of that lane capacity.
template <typename T, int D, bool FP8, int COMPACT>
int launch_tma(const DkPagedAttnArgs& a, const DkPlan& pl, DecodeParams& p, int dev, cudaStream_t stream) {
  using Shape = std::conditional_t<FP8, TmaShapeFp8<D>, TmaShape<D>>;
  static bool attr_done[kMaxDevices] = {false};
  static int occ[kMaxDevices] = {0};
  auto kernel =
      paged_decode_tma_kernel<T, D, Shape::kStages, Shape::kWarps, FP8, Shape::kSlices, Shape::kMinCtas, COMPACT>;
  const int smem = Shape::Cfg::kSmemBytes;
  cudaError_t e = ensure_smem_attr(kernel, smem, dev, attr_done);
  if (e != cudaSuccess)
    return fail_cuda(e, FP8 ? "cudaFuncSetAttribute(fp8 partition kernel)" : "cudaFuncSetAttribute(partition kernel)");
  dim3 grid(static_cast<unsigned>(pl.num_ctas));
  if (COMPACT != 0) {
    // A fitted partition size puts every item in one wave when the lengths
    // allow it, and one wave of CTAs runs them; the CTAs loop over the items
    // when they do not.
    const bool fit = pl.fit_min_partition > 0;
    grid.x = compact_grid(kernel, Shape::Cfg::kThreads, smem, dev, pl.num_ctas, p.persistent || fit ? 1 : kCompactWaves,
                          occ);
    if (fit && dev >= 0 && dev < kMaxDevices && occ[dev] > 0) p.fit_slots = occ[dev] * num_sms(dev);
  }
  CUtensorMap kmap, vmap;
  if (int r = build_maps<D>(a, p, dev, &kmap, &vmap)) return r;
  e = launch_pdl(kernel, grid, dim3(Shape::Cfg::kThreads), smem, stream, kmap, vmap, p);
  if (e != cudaSuccess) return fail_cuda(e, FP8 ? "fp8 partition kernel launch" : "partition kernel launch");
  return 0;
}

template <typename T, int D>
int launch_typed(const DkPagedAttnArgs& a, const DkPlan& pl, DecodeParams& p, int dev, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(pl.num_ctas));  // 1-D, sequence-major (cta_coords)
  cudaError_t e;
  if (pl.path == DK_PATH_TMA_MMA && p.kv_fp8) {
    if constexpr (D >= 128) {  // e4m3 rows of at least one 128-byte block (the planner's rule)
      const int r = !p.compact ? launch_tma<T, D, true, 0>(a, pl, p, dev, stream)
                    : compact_per_lane(a.num_seqs) == kCompactSmallPerLane
                        ? launch_tma<T, D, true, kCompactSmallPerLane>(a, pl, p, dev, stream)
                        : launch_tma<T, D, true, kCompactPerLane>(a, pl, p, dev, stream);
      if (r) return r;
    } else {
      return fail(1, "internal: fp8 TMA path planned for head_dim %d", D);
    }
  } else if (pl.path == DK_PATH_TMA_MMA) {
    const int r = !p.compact ? launch_tma<T, D, false, 0>(a, pl, p, dev, stream)
                  : compact_per_lane(a.num_seqs) == kCompactSmallPerLane
                      ? launch_tma<T, D, false, kCompactSmallPerLane>(a, pl, p, dev, stream)
                      : launch_tma<T, D, false, kCompactPerLane>(a, pl, p, dev, stream);
    if (r) return r;
  } else if (p.kv_fp8) {
    auto kernel = paged_decode_simt_kernel<T, D, uint8_t>;
    e = launch_pdl(kernel, grid, dim3(kSimtThreads), SimtConfig<D>::kSmemBytes, stream, p);
    if (e != cudaSuccess) return fail_cuda(e, "fp8 partition kernel launch (CUDA-core path)");
  } else {
    auto kernel = paged_decode_simt_kernel<T, D>;
    e = launch_pdl(kernel, grid, dim3(kSimtThreads), SimtConfig<D>::kSmemBytes, stream, p);
    if (e != cudaSuccess) return fail_cuda(e, "partition kernel launch (CUDA-core path)");
  }
  if (pl.split && p.merge_counters == nullptr) {
    const dim3 mgrid(static_cast<unsigned>(a.num_q_heads), static_cast<unsigned>(a.num_seqs));
    e = launch_pdl(merge_partitions_kernel<T, D>, mgrid, dim3(kMergeThreads), 0, stream, p);
    if (e != cudaSuccess) return fail_cuda(e, "merge kernel launch");
  }
  return 0;
}

// Receive slots of a head all-gather fused into the decode's output stores.
struct PeerOutputs {
  const DkPeerGatherArgs* g;
};

int launch(const DkPagedAttnArgs& a, const DkPlan& pl, int dev, cudaStream_t stream, bool lse_mode = false,
           const PeerOutputs* peer = nullptr) {
  if (1LL * pl.num_partitions * a.num_kv_heads * a.num_seqs > INT_MAX)
    return fail(1, "paged_attention_decode: %d partitions x %d KV heads x %d sequences exceed one grid", pl.num_partitions,
                a.num_kv_heads, a.num_seqs);
  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  p.lse_mode = lse_mode ? 1 : 0;
  p.out = a.out;
  p.q = a.q;
  p.k_cache = a.k_cache;
  p.v_cache = a.v_cache;
  p.block_tables = a.block_tables;
  p.seq_lens = a.seq_lens;
  p.tmp_out = pl.split ? a.tmp_out : nullptr;
  p.max_logits = pl.split ? a.max_logits : nullptr;
  p.exp_sums = pl.split ? a.exp_sums : nullptr;
  p.merge_counters = pl.split && pl.launches == 1 ? a.merge_counters : nullptr;
  p.q_stride_seq = a.q_stride_seq;
  p.q_stride_head = a.q_stride_head;
  p.out_stride_seq = a.out_stride_seq;
  p.out_stride_head = a.out_stride_head;
  p.k_stride_block = a.k_stride_block;
  p.k_stride_token = a.k_stride_token;
  p.k_stride_head = a.k_stride_head;
  p.v_stride_block = a.v_stride_block;
  p.v_stride_token = a.v_stride_token;
  p.v_stride_head = a.v_stride_head;
  p.bt_stride = a.bt_stride;
  p.num_seqs = a.num_seqs;
  p.num_q_heads = a.num_q_heads;
  p.num_kv_heads = a.num_kv_heads;
  p.group = a.num_q_heads / a.num_kv_heads;
  p.max_seq_len = a.max_seq_len;
  p.block_size = a.block_size;
  p.num_blocks = a.num_blocks;
  p.bs_log2 = ilog2(a.block_size);
  p.rows_log2 = std::min(p.bs_log2, ilog2(pl.path == DK_PATH_TMA_MMA && a.kv_fp8 ? tma_tile_fp8(a.head_dim)
                                                                               : tma_tile(a.head_dim)));
  p.partition_size = pl.partition_size;
  p.num_partitions = pl.num_partitions;
  p.ws_partitions = pl.split ? a.max_partitions : 1;
  p.split = pl.split;
  p.kv_fp8 = a.kv_fp8;
  // Compact grid (compact_coords) when most CTAs of the dense grid may have no
  // tokens -- a sequence may span many partitions -- and few enough sequences
  // that every CTA's warp scan of the lengths stays short; its CTAs pay that
  // scan before their first loads.  With DK_FLAG_PERSISTENT, whenever the
  // device fits the partition size (fit_partition_size), and by default:
  // * e4m3 caches, 4 waves of CTAs: the consumers' math bounds a CTA (c4f8
  //   80.7 -> ~73 us with the planned size);
  // * 16-bit caches with at most one (sequence, KV head) pair per SM, one
  //   wave (the persistent grid): c4 78.2 -> 76.5 us at the planned 1728
  //   tokens, where the dense grid's 2432 CTAs hold 323 live items.  (4 waves
  //   measured slower on an earlier kernel, c4 85 -> 89 us; HBM bounds a
  //   16-bit CTA, and the empty CTAs' dispatch is what the one wave saves.)
  const bool persistent = (a.flags & DK_FLAG_PERSISTENT) != 0;
  const bool sparse = pl.num_partitions >= kCompactMinPartitions && a.num_seqs > 1;
  const bool one_wave16 =
      !a.kv_fp8 && sparse && fit_shape(a.num_seqs, a.num_kv_heads, a.max_seq_len, num_sms(dev));
  p.compact = pl.path == DK_PATH_TMA_MMA && a.num_seqs <= kCompactMaxSeqs &&
              (persistent || pl.fit_min_partition > 0 || (a.kv_fp8 && sparse) || one_wave16);
  p.persistent = p.compact && (persistent || one_wave16);
  p.fit_min_partition = pl.fit_min_partition;
  p.fit_gran = pl.path == DK_PATH_TMA_MMA && a.kv_fp8 ? tma_tile_fp8(a.head_dim) : DK_TILE_TOKENS;
  p.fit_slots = 0;  // set at launch from the kernel's occupancy
  p.scale_log2 = a.scale * (a.kv_fp8 ? a.k_scale : 1.0f) * kLog2e;
  p.v_scale = a.kv_fp8 ? a.v_scale : 1.0f;
  if (peer != nullptr) {
    const DkPeerGatherArgs& g = *peer->g;
    for (int r = 0; r < g.world; ++r) p.peer_recv[r] = g.recv[r];
    p.peer_state = g.state;
    p.peer_world = g.world;
    p.peer_q_heads = g.heads_per_rank * g.world;
    p.peer_head0 = g.rank * g.heads_per_rank;
    p.peer_slot_elems = static_cast<int64_t>(g.num_seqs) * p.peer_q_heads * g.head_dim;
  }
  const bool bf16 = a.dtype == DK_DTYPE_BFLOAT16;
  switch (a.head_dim) {
    case 64:
      return bf16 ? launch_typed<__nv_bfloat16, 64>(a, pl, p, dev, stream) : launch_typed<__half, 64>(a, pl, p, dev, stream);
    case 128:
      return bf16 ? launch_typed<__nv_bfloat16, 128>(a, pl, p, dev, stream)
                  : launch_typed<__half, 128>(a, pl, p, dev, stream);
    default:
      return bf16 ? launch_typed<__nv_bfloat16, 256>(a, pl, p, dev, stream)
                  : launch_typed<__half, 256>(a, pl, p, dev, stream);
  }
}

// ---------------------------------------------------------------------------
// Scratch for dk_paged_attention_decode_noalloc: the split-K partials of
// callers that cannot allocate.  File-scope, so every GPU that loads this
// library holds it until the process exits.  Host code must not pass the
// symbol itself to a kernel (on the host it is only a stand-in); the device
// address comes from cudaGetSymbolAddress, once per device.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_noalloc_scratch[DK_NOALLOC_SCRATCH_BYTES / sizeof(float)];
// Merge counters of the no-allocation path.  A call that completes leaves the
// ones it used at zero, but one whose bounded wait gave up may not (its CTA
// skips the rest of its items), so every call that uses them clears its range
// with cudaMemsetAsync on its stream first.  Calls with more (sequence, KV
// head) pairs use the separate merge kernel.
constexpr int kNoallocCounters = 1 << 18;
static __device__ __align__(256) int g_noalloc_counters[kNoallocCounters];

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {nullptr};
int* g_noalloc_ctr[kMaxDevices] = {nullptr};

// Device addresses of the scratch and the counters on `dev` (the current
// device), looked up on the first call for that device.
int noalloc_scratch(int dev, float** out, int** counters) {
  if (dev < 0 || dev >= kMaxDevices) return fail(1, "device %d out of range for the no-allocation scratch", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return fail_cuda(e, "cudaGetSymbolAddress(no-allocation scratch)");
    void* c = nullptr;
    e = cudaGetSymbolAddress(&c, g_noalloc_counters);
    if (e != cudaSuccess || c == nullptr) return fail_cuda(e, "cudaGetSymbolAddress(no-allocation counters)");
    g_noalloc_ctr[dev] = static_cast<int*>(c);
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  *counters = g_noalloc_ctr[dev];
  return 0;
}

// ---------------------------------------------------------------------------
// Merge of partials over disjoint token ranges
// ---------------------------------------------------------------------------
int validate_lse_merge(const DkLseMergeArgs* a) {
  if (a == nullptr) return fail(1, "dk_merge_lse: args is NULL");
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256)
    return fail(1, "head_dim must be 64, 128 or 256, got %d", a->head_dim);
  if (a->num_parts < 1 || a->num_seqs < 0 || a->num_q_heads <= 0)
    return fail(1, "dk_merge_lse: num_parts must be >= 1, num_seqs >= 0, num_q_heads > 0");
  if (!a->out_partial && a->dtype != DK_DTYPE_FLOAT16 && a->dtype != DK_DTYPE_BFLOAT16)
    return fail(1, "dk_merge_lse: out must be float16 or bfloat16 (dtype code %d)", a->dtype);
  const int64_t rows = static_cast<int64_t>(a->num_seqs) * a->num_q_heads * (a->head_dim + 4);
  if (a->num_parts > 1 && a->part_stride < rows) return fail(1, "dk_merge_lse: part_stride overlaps the parts");
  if (a->num_seqs == 0) return 0;
  if (!a->parts || !a->out) return fail(1, "dk_merge_lse: NULL pointer");
  if (a->out_stride_seq < 0 || a->out_stride_head < 0) return fail(1, "dk_merge_lse: negative stride");
  return 0;
}

template <int D>
int launch_lse_merge(const DkLseMergeArgs& a, cudaStream_t stream) {
  LseMergeParams p;
  p.parts = a.parts;
  p.part_stride = a.part_stride;
  p.out = a.out;
  p.out_stride_seq = a.out_stride_seq;
  p.out_stride_head = a.out_stride_head;
  p.num_parts = a.num_parts;
  p.num_seqs = a.num_seqs;
  p.num_q_heads = a.num_q_heads;
  p.out_lse = a.out_partial;
  const long long pairs = static_cast<long long>(a.num_seqs) * a.num_q_heads;
  const dim3 grid(static_cast<unsigned>((pairs + kLseMergeThreads / 32 - 1) / (kLseMergeThreads / 32)));
  if (a.out_partial || a.dtype == DK_DTYPE_FLOAT16)
    merge_lse_kernel<__half, D><<<grid, kLseMergeThreads, 0, stream>>>(p);
  else
    merge_lse_kernel<__nv_bfloat16, D><<<grid, kLseMergeThreads, 0, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : fail_cuda(e, "LSE merge kernel launch");
}

// ---------------------------------------------------------------------------
// Peer-memory exchange of sequence-shard partials
// ---------------------------------------------------------------------------
int validate_peer_exchange(const DkPeerExchangeArgs* a) {
  if (a == nullptr) return fail(1, "dk_exchange_merge_lse: args is NULL");
  if (a->world < 1 || a->world > DK_MAX_PEERS || a->rank < 0 || a->rank >= a->world)
    return fail(1, "dk_exchange_merge_lse: need 0 <= rank < world <= %d", DK_MAX_PEERS);
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256)
    return fail(1, "head_dim must be 64, 128 or 256, got %d", a->head_dim);
  if (a->dtype != DK_DTYPE_FLOAT16 && a->dtype != DK_DTYPE_BFLOAT16)
    return fail(1, "dk_exchange_merge_lse: out must be float16 or bfloat16 (dtype code %d)", a->dtype);
  if (a->num_seqs < 0 || a->num_q_heads <= 0) return fail(1, "dk_exchange_merge_lse: bad sizes");
  if (!a->partial || !a->state || !a->out) return fail(1, "dk_exchange_merge_lse: NULL pointer");
  if (!aligned(a->partial, 16)) return fail(1, "dk_exchange_merge_lse: partial must be 16-byte aligned");
  for (int r = 0; r < a->world; ++r) {
    if (!a->recv[r] || !a->flags[r]) return fail(1, "dk_exchange_merge_lse: NULL peer pointer for rank %d", r);
    if (!aligned(a->recv[r], 16) || !aligned(a->flags[r], 4))
      return fail(1, "dk_exchange_merge_lse: receive buffers must be 16-byte aligned");
  }
  return 0;
}

template <int D>
int launch_peer_exchange(const DkPeerExchangeArgs& a, int dev, cudaStream_t stream) {
  PeerExchangeParams p;
  std::memset(&p, 0, sizeof(p));
  p.partial = a.partial;
  for (int r = 0; r < a.world; ++r) {
    p.recv[r] = a.recv[r];
    p.flags[r] = a.flags[r];
  }
  p.state = a.state;
  p.out = a.out;
  p.out_stride_seq = a.out_stride_seq;
  p.out_stride_head = a.out_stride_head;
  p.block_floats = static_cast<int64_t>(a.num_seqs) * a.num_q_heads * (D + 4);
  p.rank = a.rank;
  p.world = a.world;
  p.num_seqs = a.num_seqs;
  p.num_q_heads = a.num_q_heads;
  p.wait_limit_ns = (a.wait_limit_ms ? a.wait_limit_ms : 2000u) * 1000000ull;
  // at most two CTAs per SM: every CTA must be resident while they wait on one another's flags
  const long long pairs = static_cast<long long>(a.num_seqs) * a.num_q_heads;
  const long long want = std::max<long long>(std::max<long long>(1, (pairs + 7) / 8),
                                             (p.block_floats / 4 + kExchangeThreads - 1) / kExchangeThreads);
  const dim3 grid(static_cast<unsigned>(std::min<long long>(want, 2LL * num_sms(dev))));
  const cudaError_t e = a.dtype == DK_DTYPE_BFLOAT16
                            ? launch_pdl(peer_exchange_merge_kernel<__nv_bfloat16, D>, grid, dim3(kExchangeThreads), 0,
                                         stream, p)
                            : launch_pdl(peer_exchange_merge_kernel<__half, D>, grid, dim3(kExchangeThreads), 0, stream, p);
  return e == cudaSuccess ? 0 : fail_cuda(e, "peer exchange kernel launch");
}

int validate_peer_gather(const DkPeerGatherArgs* a, bool need_local = true) {
  if (a == nullptr) return fail(1, "dk_gather_heads: args is NULL");
  if (a->world < 1 || a->world > DK_MAX_PEERS || a->rank < 0 || a->rank >= a->world)
    return fail(1, "dk_gather_heads: need 0 <= rank < world <= %d", DK_MAX_PEERS);
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256)
    return fail(1, "head_dim must be 64, 128 or 256, got %d", a->head_dim);
  if (a->dtype != DK_DTYPE_FLOAT16 && a->dtype != DK_DTYPE_BFLOAT16)
    return fail(1, "dk_gather_heads: dtype must be float16 or bfloat16 (code %d)", a->dtype);
  if (a->num_seqs < 0 || a->heads_per_rank <= 0) return fail(1, "dk_gather_heads: bad sizes");
  const bool rows = a->num_seqs > 0;  // with no rows only the flags move (local and out may be NULL)
  if ((rows && need_local && !a->local) || !a->state || (rows && !a->out))
    return fail(1, "dk_gather_heads: NULL pointer");
  if ((rows && need_local && (!aligned(a->local, 16) || a->local_stride_seq % 8 || a->local_stride_head % 8)) ||
      !aligned(a->out, 16) || a->out_stride_seq % 8 || a->out_stride_head % 8)
    return fail(1, "dk_gather_heads: local and out rows must start on 16-byte boundaries");
  for (int r = 0; r < a->world; ++r) {
    if (!a->recv[r] || !a->flags[r]) return fail(1, "dk_gather_heads: NULL peer pointer for rank %d", r);
    if (!aligned(a->recv[r], 16) || !aligned(a->flags[r], 4))
      return fail(1, "dk_gather_heads: receive buffers must be 16-byte aligned");
  }
  return 0;
}

int launch_peer_gather(const DkPeerGatherArgs& a, int dev, cudaStream_t stream, bool push = true) {
  PeerGatherParams p;
  std::memset(&p, 0, sizeof(p));
  p.local = push ? static_cast<const uint16_t*>(a.local) : nullptr;  // nullptr: the decode already pushed
  p.local_stride_seq = a.local_stride_seq;
  p.local_stride_head = a.local_stride_head;
  for (int r = 0; r < a.world; ++r) {
    p.recv[r] = static_cast<uint16_t*>(a.recv[r]);
    p.flags[r] = a.flags[r];
  }
  p.state = a.state;
  p.out = static_cast<uint16_t*>(a.out);
  p.out_stride_seq = a.out_stride_seq;
  p.out_stride_head = a.out_stride_head;
  p.num_seqs = a.num_seqs;
  p.heads_per_rank = a.heads_per_rank;
  p.num_q_heads = a.heads_per_rank * a.world;
  p.head_dim = a.head_dim;
  p.slot_elems = static_cast<int64_t>(a.num_seqs) * p.num_q_heads * a.head_dim;
  p.rank = a.rank;
  p.world = a.world;
  p.wait_limit_ns = (a.wait_limit_ms ? a.wait_limit_ms : 2000u) * 1000000ull;
  // at most two CTAs per SM: every CTA must be resident while they wait on one another's flags
  const long long chunks = p.slot_elems / 8;
  const long long want = std::max<long long>(1, (chunks + kExchangeThreads - 1) / kExchangeThreads);
  const dim3 grid(static_cast<unsigned>(std::min<long long>(want, 2LL * num_sms(dev))));
  const cudaError_t e = launch_pdl(peer_gather_kernel, grid, dim3(kExchangeThreads), 0, stream, p);
  return e == cudaSuccess ? 0 : fail_cuda(e, "peer gather kernel launch");
}

// ---------------------------------------------------------------------------
// Paged-KV write
// ---------------------------------------------------------------------------
int validate_cache_write(const DkCacheWriteArgs* a) {
  if (a == nullptr) return fail(1, "dk_reshape_and_cache: args is NULL");
  if (a->dtype != DK_DTYPE_FLOAT16 && a->dtype != DK_DTYPE_BFLOAT16)
    return fail(1, "reshape_and_cache: key/value must be float16 or bfloat16 (dtype code %d)", a->dtype);
  if (a->cache_dtype != a->dtype && a->cache_dtype != DK_DTYPE_FP8_E4M3)
    return fail(1, "reshape_and_cache: cache dtype must match key/value or be fp8 e4m3 (code %d)", a->cache_dtype);
  if (a->num_tokens < 0) return fail(1, "reshape_and_cache: num_tokens must be non-negative");
  if (a->num_kv_heads <= 0 || a->head_dim <= 0 || a->block_size <= 0 || a->num_blocks <= 0)
    return fail(1, "reshape_and_cache: num_kv_heads, head_dim, block_size and num_blocks must be positive");
  if (a->cache_dtype == DK_DTYPE_FP8_E4M3 &&
      !(a->k_scale > 0.0f && a->v_scale > 0.0f && a->k_scale < INFINITY && a->v_scale < INFINITY))
    return fail(1, "reshape_and_cache: fp8 scales must be positive and finite");
  if (a->num_tokens == 0) return 0;
  if (!a->key || !a->value || !a->key_cache || !a->value_cache || !a->slot_mapping)
    return fail(1, "reshape_and_cache: NULL tensor pointer");
  const int64_t strides[10] = {a->key_stride_token, a->key_stride_head, a->value_stride_token, a->value_stride_head,
                               a->k_stride_block,   a->k_stride_token,  a->k_stride_head,      a->v_stride_block,
                               a->v_stride_token,   a->v_stride_head};
  for (int64_t st : strides) {
    if (st < 0) return fail(1, "reshape_and_cache: negative stride");
  }
  return 0;
}

template <typename T>
int launch_cache_write(const DkCacheWriteArgs& a, cudaStream_t stream) {
  CacheWriteParams p;
  p.key = a.key;
  p.value = a.value;
  p.key_cache = a.key_cache;
  p.value_cache = a.value_cache;
  p.slot_mapping = a.slot_mapping;
  p.key_stride_token = a.key_stride_token;
  p.key_stride_head = a.key_stride_head;
  p.value_stride_token = a.value_stride_token;
  p.value_stride_head = a.value_stride_head;
  p.k_stride_block = a.k_stride_block;
  p.k_stride_token = a.k_stride_token;
  p.k_stride_head = a.k_stride_head;
  p.v_stride_block = a.v_stride_block;
  p.v_stride_token = a.v_stride_token;
  p.v_stride_head = a.v_stride_head;
  p.num_slots = static_cast<int64_t>(a.num_blocks) * a.block_size;
  p.num_kv_heads = a.num_kv_heads;
  p.head_dim = a.head_dim;
  p.block_size = a.block_size;
  p.k_scale = a.k_scale;
  p.v_scale = a.v_scale;
  const bool fp8 = a.cache_dtype == DK_DTYPE_FP8_E4M3;
  // 8-element steps when every row start is aligned for them
  const size_t cache_esz = fp8 ? 1 : 2;
  bool vec = a.head_dim % 8 == 0 && aligned(a.key, 16) && aligned(a.value, 16) &&
             aligned(a.key_cache, 8 * cache_esz) && aligned(a.value_cache, 8 * cache_esz);
  const int64_t strides[10] = {a.key_stride_token, a.key_stride_head, a.value_stride_token, a.value_stride_head,
                               a.k_stride_block,   a.k_stride_token,  a.k_stride_head,      a.v_stride_block,
                               a.v_stride_token,   a.v_stride_head};
  for (int64_t st : strides) vec = vec && st % 8 == 0;
  const dim3 grid(static_cast<unsigned>(a.num_tokens));
  const dim3 block(kCacheWriteThreads);
  if (fp8) {
    if (vec)
      reshape_and_cache_kernel<T, true, 8><<<grid, block, 0, stream>>>(p);
    else
      reshape_and_cache_kernel<T, true, 1><<<grid, block, 0, stream>>>(p);
  } else {
    if (vec)
      reshape_and_cache_kernel<T, false, 8><<<grid, block, 0, stream>>>(p);
    else
      reshape_and_cache_kernel<T, false, 1><<<grid, block, 0, stream>>>(p);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : fail_cuda(e, "reshape_and_cache kernel launch");
}

}  // namespace
}  // namespace dkb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

int dk_paged_attention_decode(const DkPagedAttnArgs* args, dk_stream_t stream) {
  if (int e = dkb::validate(args)) return e;
  if (args->num_seqs == 0) return 0;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return dkb::fail_cuda(ce, "cudaGetDevice");
  DkPlan pl;
  dkb::make_plan(*args, dev, &pl);
  if (pl.split && args->max_partitions < pl.num_partitions)
    return dkb::fail(1, "split-K workspace too small: %d partitions needed", pl.num_partitions);
  return dkb::launch(*args, pl, dev, reinterpret_cast<cudaStream_t>(stream));
}

int dk_paged_attention_decode_noalloc(const DkPagedAttnArgs* args, dk_stream_t stream) {
  if (int e = dkb::validate(args)) return e;
  if (args->max_partitions != 0 || args->tmp_out || args->max_logits || args->exp_sums)
    return dkb::fail(1, "dk_paged_attention_decode_noalloc takes no workspace: set max_partitions to 0 and the "
                        "workspace pointers to NULL");
  if (args->num_seqs == 0) return 0;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return dkb::fail_cuda(ce, "cudaGetDevice");
  // Plan as if the caller had allocated the planner's full workspace, so the
  // partitioning (and the result) is the same as dk_paged_attention_decode's.
  DkPagedAttnArgs a = *args;
  a.max_partitions = INT_MAX;
  a.merge_counters = nullptr;
  DkPlan pl;
  dkb::make_plan(a, dev, &pl);
  const size_t row_bytes = static_cast<size_t>(a.num_seqs) * a.num_q_heads * (a.head_dim + 2) * sizeof(float);
  if (pl.fit_min_partition > 0 && row_bytes * pl.num_partitions > DK_NOALLOC_SCRATCH_BYTES) {
    // A fitted size's rows (down to its floor) do not fit the scratch, the
    // planned size's do: raise the floor to what the scratch holds.
    const size_t fit_rows = DK_NOALLOC_SCRATCH_BYTES / row_bytes;
    if (fit_rows >= static_cast<size_t>(dkb::ceil_div(a.max_seq_len, pl.partition_size))) {
      a.max_partitions = static_cast<int>(fit_rows);
      dkb::make_plan(a, dev, &pl);
    }
  }
  a.max_partitions = 0;
  if (pl.split) {
    const size_t rows = static_cast<size_t>(a.num_seqs) * a.num_q_heads * pl.num_partitions;
    const size_t need = rows * (static_cast<size_t>(a.head_dim) + 2) * sizeof(float);
    if (need > DK_NOALLOC_SCRATCH_BYTES)
      return dkb::fail(1,
                       "dk_paged_attention_decode_noalloc: this call needs %zu bytes of split-K scratch "
                       "(%d sequences x %d query heads x %d partitions x (head_dim + 2) floats) but the static "
                       "scratch holds %u bytes; call dk_paged_attention_decode with a caller-allocated workspace",
                       need, a.num_seqs, a.num_q_heads, pl.num_partitions, DK_NOALLOC_SCRATCH_BYTES);
    float* base = nullptr;
    int* counters = nullptr;
    if (int e = dkb::noalloc_scratch(dev, &base, &counters)) return e;
    a.tmp_out = base;
    a.max_logits = base + rows * a.head_dim;
    a.exp_sums = a.max_logits + rows;
    a.max_partitions = pl.num_partitions;
    const long long pairs = static_cast<long long>(a.num_seqs) * a.num_kv_heads;
    if (pairs <= dkb::kNoallocCounters) {
      a.merge_counters = counters;  // one launch when the merge is small
      // Same partitions (the rows hold the planned count, so neither the
      // planned size nor a fitted size's floor moves); only the merge choice
      // is re-planned.
      dkb::make_plan(a, dev, &pl);
      if (pl.launches == 1) {
        // Start from zero whatever an earlier call left behind (a wait that
        // gave up leaves its pairs' counts part-way); a memset allocates nothing.
        ce = cudaMemsetAsync(counters, 0, static_cast<size_t>(pairs) * sizeof(int),
                             reinterpret_cast<cudaStream_t>(stream));
        if (ce != cudaSuccess) return dkb::fail_cuda(ce, "cudaMemsetAsync(no-allocation merge counters)");
      }
    }
  }
  return dkb::launch(a, pl, dev, reinterpret_cast<cudaStream_t>(stream));
}

int dk_plan(const DkPagedAttnArgs* args, DkPlan* plan) {
  if (plan == nullptr) return dkb::fail(1, "dk_plan: plan is NULL");
  if (int e = dkb::validate(args)) return e;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  dkb::make_plan(*args, dev, plan);
  int count = 0;
  if (dev >= 0 && cudaGetDeviceCount(&count) == cudaSuccess && count > 0)
    plan->ctas_per_sm = dkb::plan_occupancy(*args, *plan, dev);
  else
    cudaGetLastError();
  return 0;
}

int32_t dk_num_partitions(int32_t num_seqs, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                          int32_t max_seq_len, int32_t device) {
  (void)block_size;
  if (num_seqs < 0 || max_seq_len < 0 || (head_dim != 64 && head_dim != 128 && head_dim != 256)) return -1;
  if (max_seq_len == 0) return 1;
  int dev = device;
  if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = -1;
  }
  const int hkv = num_kv_heads <= 0 ? 1 : num_kv_heads;
  const int sms = dkb::num_sms(dev);
  const int ps = dkb::desired_partition_size(num_seqs, hkv, head_dim, max_seq_len, sms);
  // rows down to the smallest size the device may fit, plus the row that
  // passes its choice to the merge kernel (the cache type and path are not
  // known here)
  if (dkb::fit_shape(num_seqs, hkv, max_seq_len, sms) && ps > dkb::kFitMinPartition)
    return dkb::ceil_div(max_seq_len, dkb::kFitMinPartition) + 1;
  return dkb::ceil_div(max_seq_len, ps);
}

int dk_paged_attention_decode_lse(const DkPagedAttnArgs* args, float* partial, dk_stream_t stream) {
  if (args == nullptr) return dkb::fail(1, "dk_paged_attention_decode_lse: args is NULL");
  DkPagedAttnArgs a = *args;
  a.out = partial;
  a.out_stride_head = a.head_dim + 4;
  a.out_stride_seq = static_cast<int64_t>(a.num_q_heads) * a.out_stride_head;
  if (int e = dkb::validate(&a)) return e;
  if (a.num_seqs == 0) return 0;
  if (!dkb::aligned(partial, 16)) return dkb::fail(1, "dk_paged_attention_decode_lse: partial must be 16-byte aligned");
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return dkb::fail_cuda(ce, "cudaGetDevice");
  DkPlan pl;
  dkb::make_plan(a, dev, &pl);
  if (pl.split && a.max_partitions < pl.num_partitions)
    return dkb::fail(1, "split-K workspace too small: %d partitions needed", pl.num_partitions);
  return dkb::launch(a, pl, dev, reinterpret_cast<cudaStream_t>(stream), /*lse_mode=*/true);
}

int dk_merge_lse(const DkLseMergeArgs* args, dk_stream_t stream) {
  if (int e = dkb::validate_lse_merge(args)) return e;
  if (args->num_seqs == 0) return 0;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (args->head_dim) {
    case 64:
      return dkb::launch_lse_merge<64>(*args, s);
    case 128:
      return dkb::launch_lse_merge<128>(*args, s);
    default:
      return dkb::launch_lse_merge<256>(*args, s);
  }
}

int dk_exchange_merge_lse(const DkPeerExchangeArgs* args, dk_stream_t stream) {
  if (int e = dkb::validate_peer_exchange(args)) return e;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return dkb::fail_cuda(ce, "cudaGetDevice");
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (args->head_dim) {
    case 64:
      return dkb::launch_peer_exchange<64>(*args, dev, s);
    case 128:
      return dkb::launch_peer_exchange<128>(*args, dev, s);
    default:
      return dkb::launch_peer_exchange<256>(*args, dev, s);
  }
}

int dk_paged_attention_decode_gather(const DkPagedAttnArgs* args, const DkPeerGatherArgs* gather,
                                     dk_stream_t stream) {
  if (args == nullptr) return dkb::fail(1, "dk_paged_attention_decode_gather: args is NULL");
  if (int e = dkb::validate_peer_gather(gather, false)) return e;
  DkPagedAttnArgs a = *args;
  if (gather->num_seqs != a.num_seqs || gather->heads_per_rank != a.num_q_heads || gather->head_dim != a.head_dim ||
      gather->dtype != a.dtype)
    return dkb::fail(1,
                     "dk_paged_attention_decode_gather: the gather's num_seqs, heads_per_rank, head_dim and dtype must "
                     "be the decode's num_seqs, num_q_heads, head_dim and dtype");
  a.out = gather->out;  // validated as a place to write; the decode's rows go to the receive slots
  a.out_stride_seq = gather->out_stride_seq;
  a.out_stride_head = gather->out_stride_head;
  if (int e = dkb::validate(&a)) return e;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return dkb::fail_cuda(ce, "cudaGetDevice");
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a.num_seqs > 0) {
    DkPlan pl;
    dkb::make_plan(a, dev, &pl);
    const dkb::PeerOutputs peer{gather};
    if (int e = dkb::launch(a, pl, dev, s, false, &peer)) return e;
  }
  return dkb::launch_peer_gather(*gather, dev, s, false);  // every rank publishes and waits, even with no rows
}

int dk_gather_heads(const DkPeerGatherArgs* args, dk_stream_t stream) {
  if (int e = dkb::validate_peer_gather(args)) return e;
  int dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess) return dkb::fail_cuda(ce, "cudaGetDevice");
  return dkb::launch_peer_gather(*args, dev, reinterpret_cast<cudaStream_t>(stream));
}

int dk_reshape_and_cache(const DkCacheWriteArgs* args, dk_stream_t stream) {
  if (int e = dkb::validate_cache_write(args)) return e;
  if (args->num_tokens == 0) return 0;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return args->dtype == DK_DTYPE_BFLOAT16 ? dkb::launch_cache_write<__nv_bfloat16>(*args, s)
                                          : dkb::launch_cache_write<__half>(*args, s);
}

const char* dk_last_error(void) { return dkb::g_last_error; }

int dk_device_wait_timeouts(int32_t device, uint32_t* count) {
  if (count == nullptr) return dkb::fail(1, "dk_device_wait_timeouts: count is NULL");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return dkb::fail_cuda(e, "cudaGetDevice");
  if (device >= 0 && device != prev && (e = cudaSetDevice(device)) != cudaSuccess)
    return dkb::fail_cuda(e, "cudaSetDevice");
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, dkb::g_wait_timeouts, sizeof(v));
  if (device >= 0 && device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return dkb::fail_cuda(e, "cudaMemcpyFromSymbol");
  *count = v;
  return 0;
}

int32_t dk_version(void) { return dkb::kVersion; }

}  // extern "C"
