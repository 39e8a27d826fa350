// Paged-KV write: the step before decode, which stores this step's new key
// and value rows into their cache slots (vLLM's reshape_and_cache_flash;
// DecodeKernels has no counterpart -- its decode reads caches vLLM wrote).
//
//   slot = slot_mapping[t]  (block * block_size + offset; < 0 = padding, skipped)
//   key_cache[slot / bs, slot % bs, h, :] = key[t, h, :]   (same for value)
//
// With an FP8 (e4m3) cache each element is stored as sat_e4m3(x / scale)
// (IEEE fp32 division, then round-to-nearest-even to e4m3, saturating to
// +-448; NaN stays NaN), the per-tensor-scale convention of vLLM's fp8 KV
// cache.
//
// HBM-bound scatter, no reuse: one CTA per token, each thread moving 8
// consecutive elements of one head row per step (16-byte loads; 16-byte
// stores into a 16-bit cache, 8-byte stores into an FP8 cache) when every
// row start is aligned for that, else one element at a time.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdint>

namespace dkb {

struct CacheWriteParams {
  const void* key;
  const void* value;
  void* key_cache;
  void* value_cache;
  const int64_t* slot_mapping;
  int64_t key_stride_token, key_stride_head, value_stride_token, value_stride_head;
  int64_t k_stride_block, k_stride_token, k_stride_head;
  int64_t v_stride_block, v_stride_token, v_stride_head;
  int64_t num_slots;  // num_blocks * block_size
  int num_kv_heads, head_dim, block_size;
  float k_scale, v_scale;  // FP8 cache: stored = sat_e4m3(x / scale)
};

constexpr int kCacheWriteThreads = 128;

template <typename T>
struct Elem;
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float f(__half x) { return __half2float(x); }
};
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 x) { return __bfloat162float(x); }
};

__device__ __forceinline__ uint8_t to_e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

// T: element type of key/value; FP8: cache holds e4m3 bytes (else T);
// VEC: elements per thread step (8, or 1 for unaligned rows).
template <typename T, bool FP8, int VEC>
__global__ void __launch_bounds__(kCacheWriteThreads) reshape_and_cache_kernel(const CacheWriteParams p) {
  const int t = blockIdx.x;
  const int64_t slot = p.slot_mapping[t];
  if (slot < 0 || slot >= p.num_slots) return;  // padding (or out of the cache)
  const int64_t blk = slot / p.block_size;
  const int64_t off = slot - blk * p.block_size;
  const int per_head = p.head_dim / VEC;
  const int per_tensor = p.num_kv_heads * per_head;
  for (int c = threadIdx.x; c < 2 * per_tensor; c += kCacheWriteThreads) {
    const bool is_v = c >= per_tensor;
    const int cc = is_v ? c - per_tensor : c;
    const int h = cc / per_head;
    const int d = (cc - h * per_head) * VEC;
    const T* src = static_cast<const T*>(is_v ? p.value : p.key) +
                   t * (is_v ? p.value_stride_token : p.key_stride_token) +
                   h * (is_v ? p.value_stride_head : p.key_stride_head) + d;
    const int64_t dst_off = blk * (is_v ? p.v_stride_block : p.k_stride_block) +
                            off * (is_v ? p.v_stride_token : p.k_stride_token) +
                            h * (is_v ? p.v_stride_head : p.k_stride_head) + d;
    if constexpr (VEC == 8) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src));
      if constexpr (FP8) {
        const T* e = reinterpret_cast<const T*>(&raw);
        const float scale = is_v ? p.v_scale : p.k_scale;
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          lo |= static_cast<uint32_t>(to_e4m3(__fdiv_rn(Elem<T>::f(e[i]), scale))) << (8 * i);
          hi |= static_cast<uint32_t>(to_e4m3(__fdiv_rn(Elem<T>::f(e[4 + i]), scale))) << (8 * i);
        }
        uint8_t* dst = static_cast<uint8_t*>(is_v ? p.value_cache : p.key_cache) + dst_off;
        *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
      } else {
        T* dst = static_cast<T*>(is_v ? p.value_cache : p.key_cache) + dst_off;
        *reinterpret_cast<uint4*>(dst) = raw;
      }
    } else {
      if constexpr (FP8) {
        const float scale = is_v ? p.v_scale : p.k_scale;
        static_cast<uint8_t*>(is_v ? p.value_cache : p.key_cache)[dst_off] =
            to_e4m3(__fdiv_rn(Elem<T>::f(*src), scale));
      } else {
        static_cast<T*>(is_v ? p.value_cache : p.key_cache)[dst_off] = *src;
      }
    }
  }
}

}  // namespace dkb
