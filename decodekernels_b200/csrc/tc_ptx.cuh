// Inline-PTX wrappers for the 5th-generation tensor cores (tcgen05) used by
// the e4m3 partition kernel: tensor-memory (TMEM) allocation, the
// kind::f8f6f4 MMA with shared-memory operand descriptors, its completion
// signal on an mbarrier, and TMEM loads / stores.  sm_100a only.
#pragma once

#include <stdint.h>

#include "dk_ptx.cuh"

namespace dkb {

// Allocate `ncols` TMEM columns (a power of two >= 32) for this CTA; the base
// address is written to `slot` in shared memory.  One full warp calls it.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Free them (the same warp, after every TMEM access of the CTA has completed).
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Order tcgen05 operations around thread synchronisation (barriers, mbarriers).
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle (the layout TMA writes
// with CU_TENSOR_MAP_SWIZZLE_128B into 1024-byte aligned boxes): start
// address, leading and stride byte offsets (16-byte units), version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f8f6f4, e4m3 x e4m3 -> f32, dense:
// c_format F32 (bit 4), A and B e4m3 (0), A major (bit 15: 0 K-major,
// 1 MN-major), B K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_e4m3(int m, int n, bool a_mn_major) {
  return (1u << 4) | (a_mn_major ? (1u << 15) : 0u) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]; issued by one thread.
__device__ __forceinline__ void umma_e4m3(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  const uint32_t z = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc), "r"(z)
      : "memory");
}

// Arrive (count 1) on `bar` once every tcgen05 MMA this thread issued so far
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 8 consecutive 32-bit columns of this thread's TMEM lane (warp-collective:
// lane i of the warp reads lane (taddr >> 16) + i).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// f16x2 -> two e4m3 bytes (low half -> low byte), round to nearest even, saturating.
__device__ __forceinline__ uint32_t f16x2_to_e4m3x2(uint32_t h) {
  uint16_t y;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(y) : "r"(h));
  return y;
}

// two floats -> two e4m3 bytes (lo -> low byte), round to nearest even, saturating.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t y;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(y) : "f"(hi), "f"(lo));
  return y;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t y;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(y) : "r"(a), "r"(b));
  return y;
}

// Two e4m3 bytes (low byte first) as two floats.
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t two_bytes) {
  const uint32_t h = e4m3x2_to_f16x2(two_bytes);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Warp-wide max of a float (order-preserving integer key, one redux).
__device__ __forceinline__ float warp_max_f32(float x) {
  int k = __float_as_int(x);
  k = k >= 0 ? k : k ^ 0x7FFFFFFF;
  k = __reduce_max_sync(0xffffffffu, k);
  return __int_as_float(k >= 0 ? k : k ^ 0x7FFFFFFF);
}

}  // namespace dkb
