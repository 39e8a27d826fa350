// Per-warp decode attention over 16-token slices of TMA-staged FP8 (e4m3)
// KV tiles: the consumer warps of the TMA partition kernel when the caches
// hold e4m3 bytes.  Same online softmax as tile_math.cuh; what differs is how
// the 8-bit rows become 16-bit mma operands, in registers, with no extra
// shared-memory pass:
//
// * S^T = K Q^T on mma.m16n8k16 (f16).  ldmatrix (b16, not transposed) gives
//   lane (g = lane/4, c = lane%4) bytes 4c..4c+3 of token row g of a 16-byte
//   column chunk.  The contraction index is permuted consistently in A and B:
//   logical columns (2c, 2c+1) are bytes (4c, 4c+1) and (2c+8, 2c+9) are
//   bytes (4c+2, 4c+3), so each half of the register converts straight into
//   one A register (cvt e4m3x2 -> f16x2), and the Q^T fragments are built
//   from q columns (4c, 4c+1) and (4c+2, 4c+3) of each 16-column block.
// * O^T += V^T P^T.  ldmatrix.trans (b16) gives lane tokens (2c, 2c+1) of
//   byte pair (2g, 2g+1) of a chunk; one byte permute regroups them into
//   (token 2c, 2c+1) pairs for d = 2g and for d = 2g+1, i.e. the A rows g and
//   g+8 of a row-permuted V^T block (row m <-> d = 2m, row m+8 <-> d = 2m+1).
//   The accumulator rows come out permuted the same way (to_red undoes it).
//
// The mma runs in f16 whatever q's type: e4m3 values are exact in f16 (the
// hardware cvt e4m3x2 -> f16x2 measured faster than an integer-op bit shuffle
// here), and a bf16 query is brought into f16 range by an exact power of two
// 2^-s taken from its largest element (s = 0 unless |q| >= 2^15), the 2^s
// going into the logit scale.  The caller folds k_scale into that scale and
// v_scale into the epilogue.
#pragma once

#include "decode_params.cuh"
#include "dk_ptx.cuh"
#include "partition_epilogue.cuh"
#include "tile_math.cuh"

namespace dkb {

template <typename T, int D>
struct WarpAttentionFp8 {
  static constexpr int MT = D / 16;   // 16-column chunks (S) = 16-row V^T blocks (PV)
  static constexpr int H = D / 128;   // 128-byte column blocks per e4m3 row
  uint32_t qf[MT][2];                 // f16 Q^T B fragments, columns permuted as above
  float m0, m1;
  float l0, l1;
  float acc[MT][4];
  float q_scale;                      // 2^s removed from q (1 for an f16 query)

  __device__ __forceinline__ void reset() {
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.0f;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[mt][j] = 0.0f;
    }
  }

  __device__ __forceinline__ void load_q_global(const DecodeParams& p, int seq, int kv_head, int lane) {
    const int qn = lane >> 2;
    const int c = lane & 3;
    const T* qrow = static_cast<const T*>(p.q) + static_cast<int64_t>(seq) * p.q_stride_seq +
                    static_cast<int64_t>(kv_head * p.group + qn) * p.q_stride_head;
    float v[MT][4];
    float mx = 0.0f;
#pragma unroll
    for (int kk = 0; kk < MT; ++kk) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[kk][j] = qn < p.group ? Conv<T>::to_f32(qrow[kk * 16 + 4 * c + j]) : 0.0f;
        mx = fmaxf(mx, fabsf(v[kk][j]));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // exact power of two keeping |q| * 2^-s below 2^15 (f16 max is 65504)
    const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFF) - 127;
    const int s = e >= 15 ? e - 14 : 0;
    const float down = __uint_as_float(static_cast<uint32_t>(127 - s) << 23);
    q_scale = __uint_as_float(static_cast<uint32_t>(127 + s) << 23);
#pragma unroll
    for (int kk = 0; kk < MT; ++kk) {
      qf[kk][0] = Conv<__half>::pack2(v[kk][0] * down, v[kk][1] * down);
      qf[kk][1] = Conv<__half>::pack2(v[kk][2] * down, v[kk][3] * down);
    }
  }

  // One 16-token slice: tile rows r0..r0+15 of the stage at `sb`, first token
  // `sub0`; tokens >= pend are masked (and their V rows cleared).
  __device__ __forceinline__ void slice(uint32_t sb, const StageGeom<H>& g, int r0, int sub0, int pend,
                                        float scale_log2, int lane) {
    const int row = r0 + (lane & 7) + (((lane >> 3) & 1) << 3);  // matrix rows: lanes 0-7, 8-15, 16-23, 24-31
    const int half = lane >> 4;                                   // 0: chunk j, 1: chunk j + 1
    const int sw = row & 7;
    const uint32_t k_base = sb + g.k_row(row);
    const uint32_t v_base = sb + g.v_row(row);

    float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float sb2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int kk = 0; kk < MT; kk += 2) {
      const int chunk = kk + half;
      uint32_t r[4];
      ldmatrix_x4(r, k_base + (chunk >> 3) * g.hstride + (((chunk & 7) ^ sw) << 4));
      // bytes (4c, 4c+1) -> A register 0/1, bytes (4c+2, 4c+3) -> A register 2/3
      uint32_t a[4];
      e4m3x4_to_f16x2x2(r[0], a[0], a[2]);
      e4m3x4_to_f16x2x2(r[1], a[1], a[3]);
      Mma<__half>::run(sa, a, qf[kk][0], qf[kk][1]);
      e4m3x4_to_f16x2x2(r[2], a[0], a[2]);
      e4m3x4_to_f16x2x2(r[3], a[1], a[3]);
      Mma<__half>::run(sb2, a, qf[kk + 1][0], qf[kk + 1][1]);
    }
    float sc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[i] = (sa[i] + sb2[i]) * scale_log2;
    const int tok_a = sub0 + (lane >> 2);
    if (tok_a >= pend) sc[0] = sc[1] = -INFINITY;
    if (tok_a + 8 >= pend) sc[2] = sc[3] = -INFINITY;

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
    if (__any_sync(0xffffffffu, al0 != 1.0f || al1 != 1.0f)) {  // skipped once the running maxima settle
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        acc[mt][0] *= al0;
        acc[mt][1] *= al1;
        acc[mt][2] *= al0;
        acc[mt][3] *= al1;
      }
    }
    const uint32_t pb0 = movmatrix_trans(Conv<__half>::pack2(p0, p1));
    const uint32_t pb1 = movmatrix_trans(Conv<__half>::pack2(p2, p3));

    if (sub0 + kSubTokens > pend) {
      // rows of tokens >= pend hold stale bytes (possibly NaN codes): clear them
      const int first_bad = r0 + (pend - sub0);
      for (int i = lane; i < kSubTokens * H * 8; i += 32) {
        const int rr = r0 + i / (H * 8);
        const int rem = i % (H * 8);
        if (rr >= first_bad) st_shared_zero16(sb + g.v_row(rr) + (rem >> 3) * g.hstride + ((rem & 7) << 4));
      }
      fence_proxy_async_smem();
      __syncwarp();
    }
#pragma unroll
    for (int mt = 0; mt < MT; mt += 2) {
      const int chunk = mt + half;
      uint32_t r[4];
      ldmatrix_x4_trans(r, v_base + (chunk >> 3) * g.hstride + (((chunk & 7) ^ sw) << 4));
      // r[i] bytes: (tok 2c, d 2g), (tok 2c, d 2g+1), (tok 2c+1, d 2g), (tok 2c+1, d 2g+1);
      // row g (d 2g) takes bytes 0 and 2, row g + 8 (d 2g+1) bytes 1 and 3
      uint32_t a[4];
      e4m3x4_to_f16x2x2(prmt(r[0], 0u, 0x3120u), a[0], a[1]);
      e4m3x4_to_f16x2x2(prmt(r[1], 0u, 0x3120u), a[2], a[3]);  // tokens 8-15
      Mma<__half>::run(acc[mt], a, pb0, pb1);
      e4m3x4_to_f16x2x2(prmt(r[2], 0u, 0x3120u), a[0], a[1]);
      e4m3x4_to_f16x2x2(prmt(r[3], 0u, 0x3120u), a[2], a[3]);
      Mma<__half>::run(acc[mt + 1], a, pb0, pb1);
    }
  }

  // K chunk pair kk, kk + 1 of one 16-row slice -> A fragments (permuted columns).
  __device__ __forceinline__ static void k_frags(uint32_t addr, uint32_t (&a0)[4], uint32_t (&a1)[4]) {
    uint32_t r[4];
    ldmatrix_x4(r, addr);
    e4m3x4_to_f16x2x2(r[0], a0[0], a0[2]);
    e4m3x4_to_f16x2x2(r[1], a0[1], a0[3]);
    e4m3x4_to_f16x2x2(r[2], a1[0], a1[2]);
    e4m3x4_to_f16x2x2(r[3], a1[1], a1[3]);
  }

  // V chunk pair mt, mt + 1 of one 16-row slice -> row-permuted V^T A fragments.
  __device__ __forceinline__ static void v_frags(uint32_t addr, uint32_t (&a0)[4], uint32_t (&a1)[4]) {
    uint32_t r[4];
    ldmatrix_x4_trans(r, addr);
    e4m3x4_to_f16x2x2(prmt(r[0], 0u, 0x3120u), a0[0], a0[1]);
    e4m3x4_to_f16x2x2(prmt(r[1], 0u, 0x3120u), a0[2], a0[3]);
    e4m3x4_to_f16x2x2(prmt(r[2], 0u, 0x3120u), a1[0], a1[1]);
    e4m3x4_to_f16x2x2(prmt(r[3], 0u, 0x3120u), a1[2], a1[3]);
  }

  // Two 16-token slices (tile rows r0..r0+31, first token sub0) with one
  // softmax update: their K chains and conversions interleave, and the
  // running max, the rescale and the exp-sum update happen once per 32
  // tokens instead of once per 16.
  __device__ __forceinline__ void slice2(uint32_t sb, const StageGeom<H>& g, int r0, int sub0, int pend,
                                         float scale_log2, int lane) {
    const int ra = r0 + (lane & 7) + (((lane >> 3) & 1) << 3);  // slice A row of this lane's ldmatrix address
    const int rb = ra + kSubTokens;                              // slice B
    const int half = lane >> 4;
    const uint32_t ka = sb + g.k_row(ra), kb = sb + g.k_row(rb);
    const uint32_t va = sb + g.v_row(ra), vb = sb + g.v_row(rb);
    const int swa = ra & 7, swb = rb & 7;

    float sA0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sA1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float sB0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sB1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int kk = 0; kk < MT; kk += 2) {
      const int chunk = kk + half;
      uint32_t aA0[4], aA1[4], aB0[4], aB1[4];
      k_frags(ka + (chunk >> 3) * g.hstride + (((chunk & 7) ^ swa) << 4), aA0, aA1);
      k_frags(kb + (chunk >> 3) * g.hstride + (((chunk & 7) ^ swb) << 4), aB0, aB1);
      Mma<__half>::run(sA0, aA0, qf[kk][0], qf[kk][1]);
      Mma<__half>::run(sB0, aB0, qf[kk][0], qf[kk][1]);
      Mma<__half>::run(sA1, aA1, qf[kk + 1][0], qf[kk + 1][1]);
      Mma<__half>::run(sB1, aB1, qf[kk + 1][0], qf[kk + 1][1]);
    }
    float sa[4], sbb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sa[i] = (sA0[i] + sA1[i]) * scale_log2;
      sbb[i] = (sB0[i] + sB1[i]) * scale_log2;
    }
    const int tok = sub0 + (lane >> 2);
    if (tok >= pend) sa[0] = sa[1] = -INFINITY;
    if (tok + 8 >= pend) sa[2] = sa[3] = -INFINITY;
    if (tok + 16 >= pend) sbb[0] = sbb[1] = -INFINITY;
    if (tok + 24 >= pend) sbb[2] = sbb[3] = -INFINITY;

    float mx0 = fmaxf(fmaxf(sa[0], sa[2]), fmaxf(sbb[0], sbb[2]));
    float mx1 = fmaxf(fmaxf(sa[1], sa[3]), fmaxf(sbb[1], sbb[3]));
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
    const float pa0 = fast_exp2(sa[0] - mn0), pa1 = fast_exp2(sa[1] - mn1);
    const float pa2 = fast_exp2(sa[2] - mn0), pa3 = fast_exp2(sa[3] - mn1);
    const float pb0 = fast_exp2(sbb[0] - mn0), pb1 = fast_exp2(sbb[1] - mn1);
    const float pb2 = fast_exp2(sbb[2] - mn0), pb3 = fast_exp2(sbb[3] - mn1);
    l0 = fmaf(l0, al0, (pa0 + pa2) + (pb0 + pb2));
    l1 = fmaf(l1, al1, (pa1 + pa3) + (pb1 + pb3));
    if (__any_sync(0xffffffffu, al0 != 1.0f || al1 != 1.0f)) {  // skipped once the running maxima settle
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        acc[mt][0] *= al0;
        acc[mt][1] *= al1;
        acc[mt][2] *= al0;
        acc[mt][3] *= al1;
      }
    }
    const uint32_t PA0 = movmatrix_trans(Conv<__half>::pack2(pa0, pa1));
    const uint32_t PA1 = movmatrix_trans(Conv<__half>::pack2(pa2, pa3));
    const uint32_t PB0 = movmatrix_trans(Conv<__half>::pack2(pb0, pb1));
    const uint32_t PB1 = movmatrix_trans(Conv<__half>::pack2(pb2, pb3));

    if (sub0 + 2 * kSubTokens > pend) {
      // rows of tokens >= pend hold stale bytes (possibly NaN codes): clear them
      const int first_bad = r0 + max(pend - sub0, 0);
      for (int i = lane; i < 2 * kSubTokens * H * 8; i += 32) {
        const int rr = r0 + i / (H * 8);
        const int rem = i % (H * 8);
        if (rr >= first_bad) st_shared_zero16(sb + g.v_row(rr) + (rem >> 3) * g.hstride + ((rem & 7) << 4));
      }
      fence_proxy_async_smem();
      __syncwarp();
    }
#pragma unroll
    for (int mt = 0; mt < MT; mt += 2) {
      const int chunk = mt + half;
      uint32_t aA0[4], aA1[4], aB0[4], aB1[4];
      v_frags(va + (chunk >> 3) * g.hstride + (((chunk & 7) ^ swa) << 4), aA0, aA1);
      v_frags(vb + (chunk >> 3) * g.hstride + (((chunk & 7) ^ swb) << 4), aB0, aB1);
      Mma<__half>::run(acc[mt], aA0, PA0, PA1);
      Mma<__half>::run(acc[mt + 1], aA1, PA0, PA1);
      Mma<__half>::run(acc[mt], aB0, PB0, PB1);
      Mma<__half>::run(acc[mt + 1], aB1, PB0, PB1);
    }
  }

  // Finish the exp-sums and store this warp's state into the merge scratch
  // (accumulator row m of block mt is column d = 16 mt + 2 (m % 8) + m / 8).
  __device__ __forceinline__ void to_red(float* red, int warps, int warp, int group, int lane) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    using Red = RedLayout<D>;
    constexpr int R = Red::kRow;
    float* red_o = Red::o(red);
    float* red_m = Red::m(red, warps);
    float* red_l = Red::l(red, warps);
    const int c0 = 2 * (lane & 3);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int h = c0 + (j & 1);
        const int d = mt * 16 + 2 * (lane >> 2) + (j >> 1);
        if (h < group) red_o[(warp * kMaxGroup + h) * R + d] = acc[mt][j];
      }
    }
    if (lane < 4) {
      red_m[warp * kMaxGroup + c0] = m0;
      red_m[warp * kMaxGroup + c0 + 1] = m1;
      red_l[warp * kMaxGroup + c0] = l0;
      red_l[warp * kMaxGroup + c0 + 1] = l1;
    }
  }
};

}  // namespace dkb
