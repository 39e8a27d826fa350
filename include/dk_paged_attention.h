/*
 * C ABI of the B200 (sm_100a) paged-attention decode library (libdk_b200.so).
 *
 * Plain pointers and sizes only: no torch types cross this boundary.  Every
 * entry point is thread-safe and allocates nothing; the caller owns every
 * buffer.  Status codes are cudaError_t values (0 = success,
 * 1 = cudaErrorInvalidValue for rejected arguments); dk_last_error() returns
 * a human-readable message for the calling thread's last failure.
 *
 * What each entry point replaces in DecodeKernels (paths inside that project):
 *
 *   dk_paged_attention_decode  <- dk::launch_paged_attention_decode<T>
 *                                 (csrc/paged_attention.cuh:309-333), the
 *                                 launcher behind the torch op
 *                                 decode_kernels::paged_attention_decode
 *                                 (csrc/ops.cu:44-144, schema :271-273)
 *   DkPagedAttnArgs            <- dk::PagedAttnParams (csrc/paged_attention.cuh:39-58)
 *                                 plus the values the launcher took as
 *                                 separate arguments (head_dim, max_seq_len)
 *                                 and the dtype the op dispatched on
 *                                 (csrc/ops.cu:17-27,139-143)
 *   dk_num_partitions          <- decode_kernels.ops.num_partitions
 *                                 (decode_kernels/ops.py:67-68), which sized
 *                                 the split-K workspace (ops.py:71-80)
 *   dk_plan                    <- the path / grid choice inside
 *                                 detail::launch (csrc/paged_attention.cuh:271-305)
 */
#ifndef DK_PAGED_ATTENTION_H_
#define DK_PAGED_ATTENTION_H_

#include <stdint.h>

#if defined(__GNUC__)
#define DK_API __attribute__((visibility("default")))
#else
#define DK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; declared here so the header needs no CUDA headers. */
typedef struct CUstream_st* dk_stream_t;

/* Element types: q, out and the K/V caches of the decode; key / value and
 * the caches of the paged-KV write (which may also store e4m3 bytes). */
enum { DK_DTYPE_FLOAT16 = 0, DK_DTYPE_BFLOAT16 = 1, DK_DTYPE_FP8_E4M3 = 2 };

/* Kernel paths reported by dk_plan. */
enum {
  DK_PATH_NONE = 0,    /* nothing to launch (num_seqs == 0) */
  DK_PATH_TMA_MMA = 1, /* TMA-staged pages + tensor-core QK^T / PV (the fast path) */
  DK_PATH_SIMT = 2     /* plain vector loads + CUDA-core math, for layouts TMA cannot describe */
};

/* Bits of DkPagedAttnArgs.flags. */
enum {
  DK_FLAG_FORCE_SIMT = 1,        /* take the CUDA-core path even when the TMA path is eligible (testing) */
  DK_FLAG_FORCE_FUSED_MERGE = 2, /* with merge counters, merge in the partition kernel whatever the merge size */
  DK_FLAG_PERSISTENT = 4         /* TMA path, <= 512 sequences: one wave of CTAs, each running every G-th
                                    live (sequence, KV head, partition) item; without it the live items
                                    are numbered densely only when a sequence may span >= 16 partitions */
};

/* Limits shared with the Python wrapper. */
#define DK_MAX_GQA_GROUP 8      /* query heads per KV head (dk::kMaxGroup) */
#define DK_TILE_TOKENS 64       /* partition sizes are multiples of this */
#define DK_REF_PARTITION_SIZE 512 /* the reference's fixed split-K partition */

/*
 * One decode call.  Shapes (row-major, strides in ELEMENTS, innermost dim
 * contiguous):
 *   q, out        [num_seqs, num_q_heads, head_dim]
 *   k/v cache     [num_blocks, block_size, num_kv_heads, head_dim] with any
 *                 strides on the first three dims (vLLM interleaved K|V,
 *                 FlashInfer NHD and HND views are read in place)
 *   block_tables  int32 [num_seqs, >= ceil(max_seq_len / block_size)], row stride bt_stride
 *   seq_lens      int32 [num_seqs], read on the device (CUDA-graph safe)
 * Split-K workspace (fp32, contiguous), used when the plan splits:
 *   tmp_out       [num_seqs, num_q_heads, max_partitions, head_dim]
 *   max_logits    [num_seqs, num_q_heads, max_partitions]
 *   exp_sums      [num_seqs, num_q_heads, max_partitions]
 * Row (seq * num_q_heads + q_head) * max_partitions + p of the workspace holds
 * partition p: its normalised partial output, its max scaled logit and its
 * exp-sum.  Set the three pointers to NULL and max_partitions to 0 when there
 * is no workspace; the call then runs single-pass.
 * Optional merge counters (no counterpart in the reference): int32
 * [num_seqs * num_kv_heads], all zero before the first call that uses them.
 * When given, the plan splits and a (sequence, KV head)'s partition rows are
 * small (<= 64 KB; any size with DK_FLAG_FORCE_FUSED_MERGE), the last
 * partition of each pair to finish merges that pair's partitions itself, so
 * the call is one kernel launch instead of two (DkPlan.launches says which).
 * Every call that completes leaves the counters zero again.  Calls that can
 * run concurrently need separate counters.  NULL keeps the separate merge
 * kernel.
 */
typedef struct DkPagedAttnArgs {
  void* out;
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const int32_t* block_tables;
  const int32_t* seq_lens;
  float* tmp_out;
  float* max_logits;
  float* exp_sums;
  int32_t* merge_counters; /* NULL, or num_seqs * num_kv_heads zeroed int32 (single-launch merge) */
  int64_t q_stride_seq, q_stride_head;
  int64_t out_stride_seq, out_stride_head;
  int64_t k_stride_block, k_stride_token, k_stride_head;
  int64_t v_stride_block, v_stride_token, v_stride_head;
  int64_t bt_stride;
  int32_t num_seqs, num_q_heads, num_kv_heads, head_dim, block_size;
  int32_t num_blocks;     /* size of the caches' first dim; ids outside [0, num_blocks) read zeros on the TMA path */
  int32_t max_seq_len;    /* host-side upper bound on seq_lens; shapes the grid (longer lengths count as this) */
  int32_t max_partitions; /* workspace capacity (tmp_out.size(2)); 0 = no workspace */
  int32_t partition_size; /* 0 = planner's choice; else a multiple of 64 tokens */
  int32_t dtype;          /* DK_DTYPE_* */
  int32_t flags;          /* DK_FLAG_* */
  float scale;            /* softmax scale, usually head_dim ** -0.5 */
  int32_t kv_fp8;         /* 1: the caches hold e4m3 bytes (K = code * k_scale, V = code * v_scale); strides and
                             alignment rules are then in bytes.  0: the caches have q's dtype */
  float k_scale, v_scale; /* FP8 caches only: positive, finite per-tensor scales */
} DkPagedAttnArgs;

/* The launch a call would make. */
typedef struct DkPlan {
  int32_t path;           /* DK_PATH_* */
  int32_t partition_size; /* tokens per partition (multiple of 64) */
  int32_t num_partitions; /* grid partitions; 1 = single pass writing out directly */
  int32_t split;          /* 1 when partitions go through the workspace and the merge kernel */
  int32_t num_ctas;       /* partition-kernel CTAs launched (including ones that exit early) */
  int32_t stages;         /* shared-memory pipeline depth of the TMA path */
  int32_t smem_bytes;     /* dynamic shared memory of the partition kernel */
  int32_t launches;       /* kernels launched by one call (1 or 2; 1 with merge counters) */
  int32_t ctas_per_sm;    /* resident partition-kernel CTAs per SM (occupancy query; 0 without a GPU) */
  int32_t fit_min_partition; /* > 0: partition_size is an upper bound; each launch fits the size on the
                                device to the batch's lengths (the smallest multiple of the kernel's tile,
                                down to this, whose live items fit one wave of resident CTAs), and
                                num_partitions covers this smallest size.  0: partition_size is used. */
} DkPlan;

/*
 * Paged-attention decode.  Launches on `stream` (asynchronous, no host sync,
 * no allocation) and returns 0, or a cudaError_t code.  Rejected arguments
 * return 1 (cudaErrorInvalidValue) without launching.  Capturable in a CUDA
 * graph: the grid depends only on host-side sizes and max_seq_len.
 */
DK_API int dk_paged_attention_decode(const DkPagedAttnArgs* args, dk_stream_t stream);

/*
 * Same decode as dk_paged_attention_decode, for callers that cannot allocate
 * device memory: no counterpart in the reference (whose wrapper always
 * allocated the split-K workspace with torch).  Examples are inference
 * runtimes and plugin hosts that hand a kernel only its inputs and outputs
 * and own every other byte of device memory, and host languages whose FFI has
 * no CUDA allocator.  Pass args with no workspace (max_partitions 0, the three
 * workspace pointers NULL); when the plan splits, the partials go to a
 * library-owned scratch array of DK_NOALLOC_SCRATCH_BYTES in device memory
 * that every GPU using this library holds until the process exits.  Calls
 * whose plan needs more scratch than that (num_seqs * num_q_heads *
 * partitions * (head_dim + 2) * 4 bytes) are rejected with status 1 and a
 * message; use dk_paged_attention_decode with your own workspace for them.
 * Nothing here calls cudaMalloc / cudaFree or any allocating routine.
 * The first call on each device looks up the scratch's device address (with
 * that device current); make that first call before any stream capture.
 * All calls share the one array: calls that can overlap on the GPU (other
 * streams, other threads) race on it.  The float partials need no clearing:
 * each call writes every scratch row it reads.  Calls with few enough
 * (sequence, KV head) pairs also use library-owned merge counters (one int32
 * per pair, at most 2^18 pairs), which must be zero when the kernel starts; a
 * completed call leaves them zero, but one whose bounded wait gave up
 * (dk_device_wait_timeouts rises) may not, so every such call first clears
 * the counters it uses with cudaMemsetAsync on `stream` (one memset node
 * before the kernel; it allocates nothing).  A later call therefore never
 * inherits a failed call's counts.
 */
#define DK_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)
DK_API int dk_paged_attention_decode_noalloc(const DkPagedAttnArgs* args, dk_stream_t stream);

/* Fill *plan with what dk_paged_attention_decode(args) would launch on the
 * current device, after the same validation.  Returns 0 or an error code. */
DK_API int dk_plan(const DkPagedAttnArgs* args, DkPlan* plan);

/*
 * Workspace partitions to allocate so the planner is never constrained:
 * ceil(max_seq_len / planned partition size).  num_kv_heads <= 0 means
 * "unknown" (sizes for the most partitions any num_kv_heads would use).
 * device < 0 means the current device.  Returns >= 1, or -1 on bad input.
 */
DK_API int32_t dk_num_partitions(int32_t num_seqs, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                          int32_t max_seq_len, int32_t device);

/*
 * Decode into fp32 partials instead of `out`: the building block of
 * sequence-sharded decode, where each GPU holds a token range of every
 * sequence (no counterpart in DecodeKernels, which runs on one GPU).
 * partial: float [num_seqs, num_q_heads, head_dim + 4], 16-byte aligned; row
 * (seq, q_head) holds the normalised output o (head_dim floats), then
 * lse = log(sum_t exp(scale * q.k_t)) over the sequence's tokens (natural
 * log; -inf and o = 0 for an empty sequence), then 3 unused floats.
 * args->out and its strides are ignored; everything else is as in
 * dk_paged_attention_decode (same planner, workspace and merge counters).
 */
DK_API int dk_paged_attention_decode_lse(const DkPagedAttnArgs* args, float* partial, dk_stream_t stream);

/*
 * Merge partials of disjoint token ranges (dk_paged_attention_decode_lse on
 * each shard):  M = max_r lse_r,  w_r = exp(lse_r - M),
 *   out = sum_r w_r o_r / sum_r w_r,  lse = M + log(sum_r w_r)
 * (zeros and lse = -inf when every part is empty).
 */
typedef struct DkLseMergeArgs {
  const float* parts;      /* num_parts partial buffers [num_seqs, num_q_heads, head_dim + 4] */
  int64_t part_stride;     /* floats from one part to the next (>= num_seqs * num_q_heads * (head_dim + 4)) */
  void* out;               /* [num_seqs, num_q_heads, head_dim] of `dtype`, or partial rows when out_partial */
  int64_t out_stride_seq;  /* elements (floats when out_partial) */
  int64_t out_stride_head;
  int32_t num_parts, num_seqs, num_q_heads, head_dim;
  int32_t dtype;           /* DK_DTYPE_FLOAT16 / DK_DTYPE_BFLOAT16 of out (ignored when out_partial) */
  int32_t out_partial;     /* 1: write merged (o, lse, pad) fp32 rows, for merging in stages */
} DkLseMergeArgs;

DK_API int dk_merge_lse(const DkLseMergeArgs* args, dk_stream_t stream);

/*
 * Exchange of sequence-shard partials over NVLink peer memory plus the merge,
 * in one kernel per GPU: the alternative to an NCCL all-gather followed by
 * dk_merge_lse.  Every GPU of the group calls it once per decode step, after
 * its dk_paged_attention_decode_lse, with the same sizes.  Memory (allocated
 * by the caller so that every GPU can address every other GPU's copy, e.g.
 * with torch.distributed symmetric memory):
 *   recv[r]   float [2][world][num_seqs * num_q_heads * (head_dim + 4)] on GPU r
 *   flags[r]  uint32 [world] on GPU r, zero before the first call
 *   state     uint32 [4] on this GPU, zero before the first call
 * The call copies `partial` into slot (call parity, rank) of every GPU's
 * receive buffer, publishes its flag on every GPU, waits (bounded by
 * wait_limit_ms; a give-up adds 1 to state[3] and the call goes on) until
 * every rank's flag has reached this call's number, and merges the world
 * slots into out [num_seqs, num_q_heads, head_dim].  The call counter lives
 * in `state`, so a captured CUDA graph replays correctly.  Concurrent calls
 * on one group need separate buffers.  world <= DK_MAX_PEERS.
 */
#define DK_MAX_PEERS 8
typedef struct DkPeerExchangeArgs {
  const float* partial;            /* this GPU's rows [num_seqs, num_q_heads, head_dim + 4] */
  float* recv[DK_MAX_PEERS];       /* receive buffers of ranks 0..world-1 as this GPU addresses them */
  uint32_t* flags[DK_MAX_PEERS];   /* flag words of ranks 0..world-1 as this GPU addresses them */
  uint32_t* state;
  void* out;
  int64_t out_stride_seq, out_stride_head;
  int32_t rank, world, num_seqs, num_q_heads, head_dim;
  int32_t dtype;                   /* DK_DTYPE_FLOAT16 / DK_DTYPE_BFLOAT16 of out */
  uint32_t wait_limit_ms;          /* 0: 2000 */
} DkPeerExchangeArgs;

DK_API int dk_exchange_merge_lse(const DkPeerExchangeArgs* args, dk_stream_t stream);

/*
 * All-gather of KV-head shards over NVLink peer memory, one kernel per GPU:
 * the alternative to an NCCL all-gather of the per-rank outputs (the gather
 * a KV-head-sharded decode needs where its consumer wants every head).  Rank
 * r holds query heads [r * heads_per_rank, (r + 1) * heads_per_rank) in
 * `local` [num_seqs, heads_per_rank, head_dim]; every GPU of the group calls
 * it once per step with the same sizes, and gets all num_q_heads =
 * world * heads_per_rank heads in out [num_seqs, num_q_heads, head_dim].
 * Memory as for dk_exchange_merge_lse:
 *   recv[r]   [2][num_seqs * num_q_heads * head_dim] elements of `dtype` on GPU r
 *   flags[r]  uint32 [world] on GPU r, zero before the first call
 *   state     uint32 [4] on this GPU, zero before the first call
 * (flags and state must not be shared with dk_exchange_merge_lse calls.)  The
 * call stores `local` into slot (call parity) of every GPU's receive buffer,
 * publishes its flag on every GPU, waits (bounded by wait_limit_ms; a
 * give-up adds 1 to state[3] and the call goes on) for every rank's flag and
 * copies the slot into `out`.  `local` and `out` rows must start on 16-byte
 * boundaries (strides multiples of 8 elements).  world <= DK_MAX_PEERS.
 */
typedef struct DkPeerGatherArgs {
  const void* local;               /* this GPU's heads [num_seqs, heads_per_rank, head_dim] of `dtype` */
  int64_t local_stride_seq, local_stride_head;
  void* recv[DK_MAX_PEERS];        /* receive buffers of ranks 0..world-1 as this GPU addresses them */
  uint32_t* flags[DK_MAX_PEERS];   /* flag words of ranks 0..world-1 as this GPU addresses them */
  uint32_t* state;
  void* out;                       /* [num_seqs, world * heads_per_rank, head_dim] of `dtype` */
  int64_t out_stride_seq, out_stride_head;
  int32_t rank, world, num_seqs, heads_per_rank, head_dim;
  int32_t dtype;                   /* DK_DTYPE_FLOAT16 / DK_DTYPE_BFLOAT16 */
  uint32_t wait_limit_ms;          /* 0: 2000 */
} DkPeerGatherArgs;

DK_API int dk_gather_heads(const DkPeerGatherArgs* args, dk_stream_t stream);

/*
 * Decode + head all-gather with the gather fused into the decode: the
 * kernels that write the output rows (partition epilogue, single-launch
 * merge or merge kernel) store them straight into slot (call parity) of
 * every rank's receive buffer over NVLink, and one small kernel then
 * publishes this rank's flag, waits for every rank's and copies the slot into
 * gather->out.  `args` is a decode of this rank's heads (args->out and its
 * strides are not used; gather->out receives all world * num_q_heads heads);
 * `gather` is as for dk_gather_heads with `local` unused (may be NULL), and
 * its num_seqs / heads_per_rank / head_dim / dtype must equal the decode's
 * num_seqs / num_q_heads / head_dim / dtype.  Every rank of the group calls
 * it once per step (also with num_seqs == 0).  Not with lse output.
 */
DK_API int dk_paged_attention_decode_gather(const DkPagedAttnArgs* args, const DkPeerGatherArgs* gather,
                                            dk_stream_t stream);

/*
 * Paged-KV write, the step before decode: no counterpart in DecodeKernels
 * (its decode reads caches that vLLM's reshape_and_cache_flash wrote); this
 * is that operation.  For every token t with slot = slot_mapping[t] in
 * [0, num_blocks * block_size):
 *   key_cache[slot / block_size, slot % block_size, h, :] = key[t, h, :]
 *   value_cache[...]                                      = value[t, h, :]
 * Negative slots (padding) and slots past the cache are skipped.  With
 * cache_dtype DK_DTYPE_FP8_E4M3 each element is stored as
 * sat_e4m3(x / scale) (IEEE fp32 division, round-to-nearest-even, saturating
 * to +-448, NaN kept), k_scale for keys and v_scale for values.  Shapes
 * (strides in ELEMENTS, head_dim contiguous):
 *   key, value          [num_tokens, num_kv_heads, head_dim]
 *   key/value_cache     [num_blocks, block_size, num_kv_heads, head_dim], any
 *                       strides on the first three dims (the decode's layouts)
 *   slot_mapping        int64 [num_tokens], on the device
 * Asynchronous on `stream`, no allocation; returns 0 or a cudaError_t code
 * (1 for rejected arguments).
 */
typedef struct DkCacheWriteArgs {
  const void* key;
  const void* value;
  void* key_cache;
  void* value_cache;
  const int64_t* slot_mapping;
  int64_t key_stride_token, key_stride_head;
  int64_t value_stride_token, value_stride_head;
  int64_t k_stride_block, k_stride_token, k_stride_head;
  int64_t v_stride_block, v_stride_token, v_stride_head;
  int32_t num_tokens, num_kv_heads, head_dim, block_size, num_blocks;
  int32_t dtype;       /* DK_DTYPE_FLOAT16 or DK_DTYPE_BFLOAT16: key and value */
  int32_t cache_dtype; /* dtype, or DK_DTYPE_FP8_E4M3 */
  float k_scale, v_scale; /* FP8 cache only: positive and finite */
} DkCacheWriteArgs;

DK_API int dk_reshape_and_cache(const DkCacheWriteArgs* args, dk_stream_t stream);

/* Message describing the calling thread's last failed call ("" if none). */
DK_API const char* dk_last_error(void);

/*
 * Bounded device-side waits that gave up since the library loaded on `device`
 * (every wait on a shared-memory barrier has a ~1 s limit; a kernel that hits
 * it records the event here and returns instead of hanging).  Synchronous.
 * Returns 0 and writes the count, or a cudaError_t code.
 */
DK_API int dk_device_wait_timeouts(int32_t device, uint32_t* count);

/* Library version, major * 10000 + minor * 100 + patch. */
DK_API int32_t dk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DK_PAGED_ATTENTION_H_ */
