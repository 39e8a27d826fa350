// Per-warp decode attention over 16-token slices of TMA-staged KV tiles
// (the consumer warps of the TMA partition kernel).
//
// A warp owns the online-softmax state of the `group` query heads of one KV
// head: the running max of two head columns per lane (log2-scaled logits),
// the lane's share of their exp-sums, and the O^T accumulator fragments.
//   S^T[16 tokens][8 heads] = K Q^T  on mma.m16n8k16 (A = K rows via ldmatrix,
//                                     B = Q^T fragments kept in registers)
//   P^T = movmatrix.trans(exp2(S^T - m))  (B fragment of the next mma)
//   O^T[D][8 heads] += V^T P^T       on mma.m16n8k16 (A = V^T via ldmatrix.trans)
// The head columns of S^T and of O^T live in the same lanes, so rescaling
// O^T when the max grows is lane-local.  bf16/fp16 in, fp32 accumulation;
// Q is used unscaled so the q.k products are exact.
#pragma once

#include "decode_params.cuh"
#include "dk_ptx.cuh"
#include "partition_epilogue.cuh"

namespace dkb {

__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
}

// Geometry of one pipeline stage: page-major, page j of a tile holds `rows`
// token rows as [K column blocks][V column blocks] x [row][128 B], 128-byte
// swizzled (a row's 16-byte chunk c sits at c ^ (row & 7)).
template <int H>
struct StageGeom {
  int rows_log2;
  int rows;
  int hstride;     // bytes between column blocks of one page (rows * 128)
  int page_bytes;  // K + V of one page (2 * H * hstride)
  __device__ __forceinline__ StageGeom(int rl) : rows_log2(rl), rows(1 << rl), hstride(rows << 7),
                                                 page_bytes(2 * H * (rows << 7)) {}
  // byte offset of tile row r's K (column block 0) within a stage
  __device__ __forceinline__ int k_row(int r) const { return (r >> rows_log2) * page_bytes + ((r & (rows - 1)) << 7); }
  __device__ __forceinline__ int v_row(int r) const { return k_row(r) + H * hstride; }
};

template <typename T, int D>
struct WarpAttention {
  static constexpr int MT = D / 16;  // 16-wide blocks of head_dim
  static constexpr int H = D / 64;   // 128-byte column blocks per row
  uint32_t qf[MT][2];                // Q^T B fragments: head lane/4, dims 2*(lane%4)..
  float m0, m1;                      // running max of columns c0, c0+1 (log2 units)
  float l0, l1;                      // this lane's share of the exp-sums
  float acc[MT][4];                  // O^T fragments

  __device__ __forceinline__ void reset() {
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.0f;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[mt][j] = 0.0f;
    }
  }

  // Q fragments straight from global memory (element loads: q needs no alignment).
  __device__ __forceinline__ void load_q_global(const DecodeParams& p, int seq, int kv_head, int lane) {
    const int qn = lane >> 2;
    const uint16_t* qrow = static_cast<const uint16_t*>(p.q) + static_cast<int64_t>(seq) * p.q_stride_seq +
                           static_cast<int64_t>(kv_head * p.group + qn) * p.q_stride_head;
#pragma unroll
    for (int kk = 0; kk < MT; ++kk) {
      const int d0 = kk * 16 + 2 * (lane & 3);
      if (qn < p.group) {
        qf[kk][0] = pack_raw16(qrow[d0], qrow[d0 + 1]);
        qf[kk][1] = pack_raw16(qrow[d0 + 8], qrow[d0 + 9]);
      } else {
        qf[kk][0] = 0u;
        qf[kk][1] = 0u;
      }
    }
  }

  // One 16-token slice: tile rows r0..r0+15 of the stage at `sb`, whose first
  // token is `sub0`; tokens >= pend are masked (and their V rows cleared).
  __device__ __forceinline__ void slice(uint32_t sb, const StageGeom<H>& g, int r0, int sub0, int pend,
                                        float scale_log2, int lane) {
    const int k_row = r0 + (lane & 7) + (((lane >> 3) & 1) << 3);  // K as A (row-major)
    const int k_chunk = lane >> 4;                                 // 0: k 0-7, 1: k 8-15
    const int v_row = r0 + (lane & 7) + ((lane >> 4) << 3);        // V^T as A (via .trans)
    const int v_chunk = (lane >> 3) & 1;                           // 0: d 0-7, 1: d 8-15
    const uint32_t k_base = sb + g.k_row(k_row);
    const int k_sw = k_row & 7;
    const uint32_t v_base = sb + g.v_row(v_row);
    const int v_sw = v_row & 7;

    // S^T = K Q^T, two accumulator chains
    float sa[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float sb2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int kk = 0; kk < MT; ++kk) {
      const int chunk = ((kk & 3) << 1) + k_chunk;
      uint32_t a[4];
      ldmatrix_x4(a, k_base + (kk >> 2) * g.hstride + ((chunk ^ k_sw) << 4));
      if (kk & 1)
        Mma<T>::run(sb2, a, qf[kk][0], qf[kk][1]);
      else
        Mma<T>::run(sa, a, qf[kk][0], qf[kk][1]);
    }
    float sc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[i] = (sa[i] + sb2[i]) * scale_log2;
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
      const int first_bad = r0 + (pend - sub0);
      for (int i = lane; i < kSubTokens * H * 8; i += 32) {
        const int row = r0 + i / (H * 8);
        const int rem = i % (H * 8);
        if (row >= first_bad) st_shared_zero16(sb + g.v_row(row) + (rem >> 3) * g.hstride + ((rem & 7) << 4));
      }
      fence_proxy_async_smem();
      __syncwarp();
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int chunk = ((mt & 3) << 1) + v_chunk;
      uint32_t a[4];
      ldmatrix_x4_trans(a, v_base + (mt >> 2) * g.hstride + ((chunk ^ v_sw) << 4));
      Mma<T>::run(acc[mt], a, pb0, pb1);
    }
  }

  // Finish the exp-sums and store this warp's state into the merge scratch.
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
  }
};

}  // namespace dkb
