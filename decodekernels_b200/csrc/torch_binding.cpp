// torch.ops.decode_kernels.paged_attention_decode: the drop-in torch op.
//
// Same schema as DecodeKernels (csrc/ops.cu:271-273), registered for the
// CUDA dispatch key (csrc/ops.cu:280-281), with the same argument checks and
// error texts (csrc/ops.cu:48-106).  Tensors are turned into plain pointers
// and element strides and handed to the C ABI (dk_paged_attention_decode in
// libdk_b200.so), which launches on the current CUDA stream of q's device.
//
// Workspace: a split-K workspace is required when max_seq_len > 512 (the
// reference's rule); a non-empty, well-formed workspace is used at any
// max_seq_len, so the per-shape planner may also split short batches.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "../../include/dk_paged_attention.h"

namespace {

void check_same(const at::Tensor& a, const at::Tensor& b, const char* what) {
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), what, ": dtype mismatch (", a.scalar_type(), " vs ",
              b.scalar_type(), ")");
  TORCH_CHECK(a.device() == b.device(), what, ": tensors must be on the same device");
}

// Checks of csrc/ops.cu:92-104.  Returns an empty string when the workspace is
// usable, else the reference's error text.
std::string workspace_problem(const at::Tensor& tmp_out, const at::Tensor& max_logits, const at::Tensor& exp_sums,
                              int64_t num_seqs, int64_t num_q_heads, int64_t head_dim, int64_t needed_parts) {
  if (!(tmp_out.scalar_type() == at::kFloat && max_logits.scalar_type() == at::kFloat &&
        exp_sums.scalar_type() == at::kFloat))
    return "split-K workspace tensors must be float32";
  if (!(tmp_out.is_contiguous() && max_logits.is_contiguous() && exp_sums.is_contiguous()))
    return "split-K workspace tensors must be contiguous";
  if (!(tmp_out.dim() == 4 && tmp_out.size(0) == num_seqs && tmp_out.size(1) == num_q_heads &&
        tmp_out.size(2) >= needed_parts && tmp_out.size(3) == head_dim))
    return "tmp_out must be [num_seqs, num_q_heads, >= ceil(max_seq_len / 512), head_dim]";
  if (!(max_logits.sizes() == exp_sums.sizes() && max_logits.dim() == 3 && max_logits.size(0) == num_seqs &&
        max_logits.size(1) == num_q_heads && max_logits.size(2) == tmp_out.size(2)))
    return "max_logits / exp_sums must be [num_seqs, num_q_heads, max_partitions]";
  if (tmp_out.size(2) > INT32_MAX) return "too many workspace partitions";
  return "";
}

// `partial` non-null: results go to fp32 rows (o, lse, pad) [n, Hq, D + 4]
// through dk_paged_attention_decode_lse and `out` is not used.
// k_scale / v_scale: dequantisation factors of e4m3 caches (uint8 or
// float8_e4m3fn tensors); a cache of q's dtype ignores them.
void decode_impl(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                 const at::Tensor& block_tables, const at::Tensor& seq_lens, double scale, int64_t max_seq_len,
                 at::Tensor& tmp_out, at::Tensor& max_logits, at::Tensor& exp_sums, at::Tensor* merge_counters,
                 at::Tensor* partial = nullptr, double k_scale = 1.0, double v_scale = 1.0, int64_t flags = 0) {
  TORCH_CHECK(q.is_cuda(), "paged_attention_decode: q must be a CUDA tensor");
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.dim() == 4,
              "k_cache and v_cache must be [num_blocks, block_size, num_kv_heads, head_dim]");
  if (partial == nullptr) {
    TORCH_CHECK(q.dim() == 3 && out.dim() == 3, "q and out must be [num_seqs, num_q_heads, head_dim]");
    check_same(q, out, "q/out");
    TORCH_CHECK(out.sizes() == q.sizes(), "out must have the same shape as q");
  } else {
    TORCH_CHECK(q.dim() == 3, "q must be [num_seqs, num_q_heads, head_dim]");
    TORCH_CHECK(partial->scalar_type() == at::kFloat && partial->is_contiguous() && partial->dim() == 3 &&
                    partial->size(0) == q.size(0) && partial->size(1) == q.size(1) &&
                    partial->size(2) == q.size(2) + 4,
                "partial must be a contiguous float32 [num_seqs, num_q_heads, head_dim + 4] tensor");
    TORCH_CHECK(partial->device() == q.device(), "partial must be on q's device");
  }
  const auto is_fp8 = [](const at::Tensor& t) {
    return t.scalar_type() == at::kByte || t.scalar_type() == at::kFloat8_e4m3fn;
  };
  const bool kv_fp8 = is_fp8(k_cache);
  if (kv_fp8) {
    TORCH_CHECK(is_fp8(v_cache), "k_cache is fp8 (e4m3) but v_cache is ", v_cache.scalar_type());
    TORCH_CHECK(k_cache.device() == q.device() && v_cache.device() == q.device(),
                "q/k_cache: tensors must be on the same device");
  } else {
    check_same(q, k_cache, "q/k_cache");
    check_same(q, v_cache, "q/v_cache");
  }
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes(), "k_cache and v_cache shapes differ");
  TORCH_CHECK(q.scalar_type() == at::kHalf || q.scalar_type() == at::kBFloat16,
              "paged_attention_decode: expected float16 or bfloat16, got ", q.scalar_type());

  const int64_t num_seqs = q.size(0);
  const int64_t num_q_heads = q.size(1);
  const int64_t head_dim = q.size(2);
  const int64_t block_size = k_cache.size(1);
  const int64_t num_kv_heads = k_cache.size(2);
  TORCH_CHECK(k_cache.size(3) == head_dim, "cache head_dim does not match q");
  TORCH_CHECK(head_dim == 64 || head_dim == 128 || head_dim == 256, "head_dim must be 64, 128 or 256, got ",
              head_dim);
  TORCH_CHECK(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, "num_q_heads must be a multiple of num_kv_heads");
  TORCH_CHECK(num_q_heads / num_kv_heads <= DK_MAX_GQA_GROUP, "GQA group size above ", DK_MAX_GQA_GROUP,
              " is not supported");
  TORCH_CHECK(q.stride(2) == 1 && (partial != nullptr || out.stride(2) == 1) && k_cache.stride(3) == 1 &&
                  v_cache.stride(3) == 1,
              "head_dim must be the contiguous (innermost) dimension");
  const int64_t vec = head_dim / 32;
  for (int d = 0; d < 3; ++d) {
    TORCH_CHECK(k_cache.stride(d) % vec == 0 && v_cache.stride(d) % vec == 0,
                "KV-cache strides must be multiples of head_dim / 32 for vectorised loads");
  }
  const int64_t kv_esz = kv_fp8 ? 1 : 2;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(k_cache.data_ptr()) % (vec * kv_esz) == 0 &&
                  reinterpret_cast<uintptr_t>(v_cache.data_ptr()) % (vec * kv_esz) == 0,
              "KV-cache pointers must be aligned to head_dim / 32 elements");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.dim() == 2 && block_tables.stride(1) == 1,
              "block_tables must be a 2-D int32 tensor with a contiguous last dimension");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.dim() == 1 && seq_lens.is_contiguous(),
              "seq_lens must be a contiguous 1-D int32 tensor");
  TORCH_CHECK(block_tables.size(0) >= num_seqs && seq_lens.size(0) >= num_seqs,
              "block_tables and seq_lens must have at least num_seqs rows");
  TORCH_CHECK(max_seq_len >= 0, "max_seq_len must be non-negative");
  TORCH_CHECK(max_seq_len <= INT32_MAX && num_seqs <= 65535 && k_cache.size(0) <= INT32_MAX,
              "paged_attention_decode: sizes exceed the supported range");

  // Workspace (csrc/ops.cu:89-106).
  const int64_t needed = (max_seq_len + DK_REF_PARTITION_SIZE - 1) / DK_REF_PARTITION_SIZE;
  int32_t max_partitions = 0;
  if (tmp_out.numel() > 0 || max_seq_len > DK_REF_PARTITION_SIZE) {
    const std::string problem =
        workspace_problem(tmp_out, max_logits, exp_sums, num_seqs, num_q_heads, head_dim, std::max<int64_t>(needed, 1));
    if (max_seq_len > DK_REF_PARTITION_SIZE) TORCH_CHECK(problem.empty(), problem);
    if (problem.empty()) {
      TORCH_CHECK(tmp_out.device() == q.device(), "split-K workspace must be on q's device");
      max_partitions = static_cast<int32_t>(tmp_out.size(2));
    }
  }
  int32_t* counters = nullptr;
  if (merge_counters != nullptr && max_partitions > 0) {
    const at::Tensor& c = *merge_counters;
    TORCH_CHECK(c.scalar_type() == at::kInt && c.is_contiguous() && c.numel() >= num_seqs * num_kv_heads,
                "merge_counters must be a contiguous int32 tensor of at least num_seqs * num_kv_heads elements");
    TORCH_CHECK(c.device() == q.device(), "merge_counters must be on q's device");
    counters = c.data_ptr<int32_t>();
  }
  if (num_seqs == 0) return;

  DkPagedAttnArgs a{};
  a.out = partial == nullptr ? out.data_ptr() : nullptr;
  a.q = q.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.block_tables = block_tables.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.tmp_out = max_partitions ? tmp_out.data_ptr<float>() : nullptr;
  a.max_logits = max_partitions ? max_logits.data_ptr<float>() : nullptr;
  a.exp_sums = max_partitions ? exp_sums.data_ptr<float>() : nullptr;
  a.merge_counters = counters;
  a.q_stride_seq = q.stride(0);
  a.q_stride_head = q.stride(1);
  a.out_stride_seq = partial == nullptr ? out.stride(0) : 0;
  a.out_stride_head = partial == nullptr ? out.stride(1) : 0;
  a.k_stride_block = k_cache.stride(0);
  a.k_stride_token = k_cache.stride(1);
  a.k_stride_head = k_cache.stride(2);
  a.v_stride_block = v_cache.stride(0);
  a.v_stride_token = v_cache.stride(1);
  a.v_stride_head = v_cache.stride(2);
  a.bt_stride = block_tables.stride(0);
  a.num_seqs = static_cast<int32_t>(num_seqs);
  a.num_q_heads = static_cast<int32_t>(num_q_heads);
  a.num_kv_heads = static_cast<int32_t>(num_kv_heads);
  a.head_dim = static_cast<int32_t>(head_dim);
  a.block_size = static_cast<int32_t>(block_size);
  a.num_blocks = static_cast<int32_t>(k_cache.size(0));
  a.max_seq_len = static_cast<int32_t>(max_seq_len);
  a.max_partitions = max_partitions;
  a.partition_size = 0;
  a.dtype = q.scalar_type() == at::kBFloat16 ? DK_DTYPE_BFLOAT16 : DK_DTYPE_FLOAT16;
  TORCH_CHECK(flags >= 0 && flags <= (DK_FLAG_FORCE_SIMT | DK_FLAG_FORCE_FUSED_MERGE | DK_FLAG_PERSISTENT),
              "paged_attention_decode: unknown flags ", flags);
  a.flags = static_cast<int32_t>(flags);
  a.scale = static_cast<float>(scale);
  a.kv_fp8 = kv_fp8 ? 1 : 0;
  a.k_scale = static_cast<float>(k_scale);
  a.v_scale = static_cast<float>(v_scale);

  const c10::cuda::OptionalCUDAGuard guard(q.device());
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  const int status =
      partial == nullptr
          ? dk_paged_attention_decode(&a, reinterpret_cast<dk_stream_t>(stream))
          : dk_paged_attention_decode_lse(&a, partial->data_ptr<float>(), reinterpret_cast<dk_stream_t>(stream));
  TORCH_CHECK(status == 0, "paged_attention_decode failed: ", dk_last_error());
}

void paged_attention_decode(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache,
                            const at::Tensor& v_cache, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                            double scale, int64_t max_seq_len, at::Tensor& tmp_out, at::Tensor& max_logits,
                            at::Tensor& exp_sums) {
  decode_impl(out, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, tmp_out, max_logits, exp_sums,
              nullptr);
}

// Same op with merge counters (int32 [num_seqs * num_kv_heads], zero before
// the first call, left zero by every completed call): when the call splits,
// the last partition of each (sequence, KV head) merges, so one kernel runs.
void paged_attention_decode_fused(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache,
                                  const at::Tensor& v_cache, const at::Tensor& block_tables,
                                  const at::Tensor& seq_lens, double scale, int64_t max_seq_len, at::Tensor& tmp_out,
                                  at::Tensor& max_logits, at::Tensor& exp_sums, at::Tensor& merge_counters) {
  decode_impl(out, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, tmp_out, max_logits, exp_sums,
              &merge_counters);
}

// Partials for sequence-sharded decode: fp32 rows (o, lse, pad).
void paged_attention_decode_lse(at::Tensor& partial, const at::Tensor& q, const at::Tensor& k_cache,
                                const at::Tensor& v_cache, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                                double scale, int64_t max_seq_len, at::Tensor& tmp_out, at::Tensor& max_logits,
                                at::Tensor& exp_sums, double k_scale, double v_scale) {
  at::Tensor unused;
  decode_impl(unused, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, tmp_out, max_logits, exp_sums,
              nullptr, &partial, k_scale, v_scale);
}

// Everything of paged_attention_decode plus optional merge counters and the
// e4m3-cache scales.
void paged_attention_decode_ext(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache,
                                const at::Tensor& v_cache, const at::Tensor& block_tables, const at::Tensor& seq_lens,
                                double scale, int64_t max_seq_len, at::Tensor& tmp_out, at::Tensor& max_logits,
                                at::Tensor& exp_sums, const c10::optional<at::Tensor>& merge_counters, double k_scale,
                                double v_scale, int64_t flags) {
  at::Tensor counters = merge_counters.has_value() ? *merge_counters : at::Tensor();
  decode_impl(out, q, k_cache, v_cache, block_tables, seq_lens, scale, max_seq_len, tmp_out, max_logits, exp_sums,
              counters.defined() ? &counters : nullptr, nullptr, k_scale, v_scale, flags);
}

// Merge partials [R, n, Hq, D + 4] (disjoint token ranges) into out: the
// attention output [n, Hq, D] (fp16 / bf16, any head / seq strides) or fp32
// partial rows [n, Hq, D + 4].
void merge_lse(at::Tensor& out, const at::Tensor& parts) {
  TORCH_CHECK(parts.is_cuda() && parts.scalar_type() == at::kFloat && parts.is_contiguous() && parts.dim() == 4,
              "parts must be a contiguous CUDA float32 [num_parts, num_seqs, num_q_heads, head_dim + 4] tensor");
  TORCH_CHECK(out.device() == parts.device(), "merge_lse: out and parts must be on the same device");
  const int64_t D = parts.size(3) - 4;
  TORCH_CHECK(out.dim() == 3 && out.size(0) == parts.size(1) && out.size(1) == parts.size(2),
              "out must be [num_seqs, num_q_heads, head_dim] or [num_seqs, num_q_heads, head_dim + 4]");
  const bool as_partial = out.scalar_type() == at::kFloat;
  TORCH_CHECK(as_partial ? (out.size(2) == D + 4 && out.is_contiguous())
                         : (out.size(2) == D && out.stride(2) == 1 &&
                            (out.scalar_type() == at::kHalf || out.scalar_type() == at::kBFloat16)),
              "merge_lse: out must be float16 / bfloat16 [.., head_dim] or contiguous float32 [.., head_dim + 4]");
  TORCH_CHECK(parts.size(0) <= INT32_MAX && parts.size(1) <= INT32_MAX && parts.size(2) <= INT32_MAX,
              "merge_lse: sizes out of range");
  DkLseMergeArgs a{};
  a.parts = parts.data_ptr<float>();
  a.part_stride = parts.stride(0);
  a.out = out.data_ptr();
  a.out_stride_seq = out.stride(0);
  a.out_stride_head = out.stride(1);
  a.num_parts = static_cast<int32_t>(parts.size(0));
  a.num_seqs = static_cast<int32_t>(parts.size(1));
  a.num_q_heads = static_cast<int32_t>(parts.size(2));
  a.head_dim = static_cast<int32_t>(D);
  a.dtype = out.scalar_type() == at::kBFloat16 ? DK_DTYPE_BFLOAT16 : DK_DTYPE_FLOAT16;
  a.out_partial = as_partial ? 1 : 0;
  const c10::cuda::OptionalCUDAGuard guard(parts.device());
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(parts.device().index()).stream();
  const int status = dk_merge_lse(&a, reinterpret_cast<dk_stream_t>(stream));
  TORCH_CHECK(status == 0, "merge_lse failed: ", dk_last_error());
}

// Paged-KV write (dk_reshape_and_cache): key/value [T, Hkv, D] into caches
// [blocks, bs, Hkv, D] (any strides on the first three dims) at slot_mapping
// (int64; negative = padding).  A uint8 / float8_e4m3fn cache stores
// sat_e4m3(x / scale).
void reshape_and_cache(const at::Tensor& key, const at::Tensor& value, at::Tensor& key_cache, at::Tensor& value_cache,
                       const at::Tensor& slot_mapping, double k_scale, double v_scale) {
  TORCH_CHECK(key.is_cuda(), "reshape_and_cache: key must be a CUDA tensor");
  TORCH_CHECK(key.dim() == 3 && value.sizes() == key.sizes(), "key and value must be [num_tokens, num_kv_heads, head_dim]");
  TORCH_CHECK(key_cache.dim() == 4 && value_cache.sizes() == key_cache.sizes(),
              "key_cache and value_cache must be [num_blocks, block_size, num_kv_heads, head_dim]");
  TORCH_CHECK(key_cache.size(2) == key.size(1) && key_cache.size(3) == key.size(2),
              "cache heads / head_dim do not match key");
  check_same(key, value, "key/value");
  TORCH_CHECK(key_cache.scalar_type() == value_cache.scalar_type(), "key_cache/value_cache: dtype mismatch");
  TORCH_CHECK(key.device() == key_cache.device() && key.device() == value_cache.device() &&
                  key.device() == slot_mapping.device(),
              "reshape_and_cache: tensors must be on the same device");
  TORCH_CHECK(key.scalar_type() == at::kHalf || key.scalar_type() == at::kBFloat16,
              "reshape_and_cache: key/value must be float16 or bfloat16, got ", key.scalar_type());
  const bool fp8 = key_cache.scalar_type() == at::kByte || key_cache.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 || key_cache.scalar_type() == key.scalar_type(),
              "reshape_and_cache: cache must have key's dtype or be uint8 / float8_e4m3fn (fp8 e4m3)");
  TORCH_CHECK(key.stride(2) == 1 && value.stride(2) == 1 && key_cache.stride(3) == 1 && value_cache.stride(3) == 1,
              "head_dim must be the contiguous (innermost) dimension");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kLong && slot_mapping.dim() == 1 && slot_mapping.is_contiguous() &&
                  slot_mapping.size(0) >= key.size(0),
              "slot_mapping must be a contiguous int64 tensor with at least num_tokens entries");
  TORCH_CHECK(key.size(0) <= INT32_MAX && key_cache.size(0) <= INT32_MAX, "reshape_and_cache: sizes out of range");
  DkCacheWriteArgs a{};
  a.key = key.data_ptr();
  a.value = value.data_ptr();
  a.key_cache = key_cache.data_ptr();
  a.value_cache = value_cache.data_ptr();
  a.slot_mapping = slot_mapping.data_ptr<int64_t>();
  a.key_stride_token = key.stride(0);
  a.key_stride_head = key.stride(1);
  a.value_stride_token = value.stride(0);
  a.value_stride_head = value.stride(1);
  a.k_stride_block = key_cache.stride(0);
  a.k_stride_token = key_cache.stride(1);
  a.k_stride_head = key_cache.stride(2);
  a.v_stride_block = value_cache.stride(0);
  a.v_stride_token = value_cache.stride(1);
  a.v_stride_head = value_cache.stride(2);
  a.num_tokens = static_cast<int32_t>(key.size(0));
  a.num_kv_heads = static_cast<int32_t>(key.size(1));
  a.head_dim = static_cast<int32_t>(key.size(2));
  a.block_size = static_cast<int32_t>(key_cache.size(1));
  a.num_blocks = static_cast<int32_t>(key_cache.size(0));
  a.dtype = key.scalar_type() == at::kBFloat16 ? DK_DTYPE_BFLOAT16 : DK_DTYPE_FLOAT16;
  a.cache_dtype = fp8 ? DK_DTYPE_FP8_E4M3 : a.dtype;
  a.k_scale = static_cast<float>(k_scale);
  a.v_scale = static_cast<float>(v_scale);
  const c10::cuda::OptionalCUDAGuard guard(key.device());
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(key.device().index()).stream();
  const int status = dk_reshape_and_cache(&a, reinterpret_cast<dk_stream_t>(stream));
  TORCH_CHECK(status == 0, "reshape_and_cache failed: ", dk_last_error());
}

}  // namespace

TORCH_LIBRARY(decode_kernels, m) {
  m.def(
      "paged_attention_decode(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
      "Tensor seq_lens, float scale, int max_seq_len, Tensor! tmp_out, Tensor! max_logits, Tensor! exp_sums) -> ()");
  m.def(
      "paged_attention_decode_fused(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
      "Tensor seq_lens, float scale, int max_seq_len, Tensor! tmp_out, Tensor! max_logits, Tensor! exp_sums, "
      "Tensor! merge_counters) -> ()");
  m.def(
      "paged_attention_decode_lse(Tensor! partial, Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
      "Tensor seq_lens, float scale, int max_seq_len, Tensor! tmp_out, Tensor! max_logits, Tensor! exp_sums, "
      "float k_scale=1.0, float v_scale=1.0) -> ()");
  m.def(
      "paged_attention_decode_ext(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
      "Tensor seq_lens, float scale, int max_seq_len, Tensor! tmp_out, Tensor! max_logits, Tensor! exp_sums, "
      "Tensor(a!)? merge_counters, float k_scale, float v_scale, int flags=0) -> ()");
  m.def("merge_lse(Tensor! out, Tensor parts) -> ()");
  m.def(
      "reshape_and_cache(Tensor key, Tensor value, Tensor! key_cache, Tensor! value_cache, Tensor slot_mapping, "
      "float k_scale, float v_scale) -> ()");
}

TORCH_LIBRARY_IMPL(decode_kernels, CUDA, m) {
  m.impl("paged_attention_decode", &paged_attention_decode);
  m.impl("paged_attention_decode_fused", &paged_attention_decode_fused);
  m.impl("reshape_and_cache", &reshape_and_cache);
  m.impl("paged_attention_decode_lse", &paged_attention_decode_lse);
  m.impl("paged_attention_decode_ext", &paged_attention_decode_ext);
  m.impl("merge_lse", &merge_lse);
}
