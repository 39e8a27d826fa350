/*
 * CPU oracle for paged-attention decode, C restatement.
 * TEST INFRASTRUCTURE, NOT PRODUCT: only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline legs load this library, as the checker or as the
 * timed CPU baseline ("port" of the reference's CPU path).
 *
 * It restates DecodeKernels' dense PyTorch oracle
 * (decode_kernels/reference.py:29-43) for one query token per sequence:
 *   token t of sequence s lives in block block_tables[s][t / bs] at offset
 *   t % bs (reference.py:15-20); scores = (q * scale) . k in fp32; probs =
 *   softmax(scores) (max-subtracted); out = probs . v; zeros for L <= 0.
 * K/V are read in place with arbitrary element strides (fp16 or bf16 bits),
 * q likewise; out is float32 [num_seqs, num_q_heads, head_dim] contiguous.
 * Work is split over (sequence, kv_head) pairs with OpenMP, or over
 * (sequence, kv_head, query head) when there are fewer pairs than threads.
 *
 * Pinned by tests/test_oracle_c.py against the numpy oracle, which is pinned
 * against the reference's golden vectors.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef struct DkOracleArgs {
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const int32_t* block_tables;
  const int32_t* seq_lens;
  float* out;
  int64_t q_stride_seq, q_stride_head;
  int64_t k_stride_block, k_stride_token, k_stride_head;
  int64_t v_stride_block, v_stride_token, v_stride_head;
  int64_t bt_stride;
  int32_t num_seqs, num_q_heads, num_kv_heads, head_dim, block_size;
  int32_t dtype; /* 0 = float16, 1 = bfloat16 */
  int32_t num_threads; /* > 0: OpenMP threads to use (whatever OMP_NUM_THREADS says); 0: OpenMP's default */
  float scale;
  int32_t threads_used; /* out: the OpenMP team size of the call */
  int32_t units;        /* out: parallel work units (pairs, or (pair, query head) when pairs < threads) */
} DkOracleArgs;

/* IEEE binary16 -> binary32, exact. */
static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do {
        ++e;
        mant <<= 1;
      } while ((mant & 0x400u) == 0);
      mant &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof(f));
  return f;
}

static float bf16_to_float(uint16_t b) {
  const uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, sizeof(f));
  return f;
}

static inline float load16(const uint16_t* p, int bf16) { return bf16 ? bf16_to_float(*p) : half_to_float(*p); }

int dk_oracle_paged_attention(DkOracleArgs* a) {
  if (!a || a->head_dim <= 0 || a->num_kv_heads <= 0 || a->num_q_heads % a->num_kv_heads) return 1;
  const int n = a->num_seqs, hq = a->num_q_heads, hkv = a->num_kv_heads, d = a->head_dim, bs = a->block_size;
  const int group = hq / hkv;
  const int bf16 = a->dtype == 1;
  const uint16_t* q = (const uint16_t*)a->q;
  const uint16_t* kc = (const uint16_t*)a->k_cache;
  const uint16_t* vc = (const uint16_t*)a->v_cache;
  const long long pairs = (long long)n * hkv;
  int status = 0;
  int threads = 1;
#ifdef _OPENMP
  threads = a->num_threads > 0 ? a->num_threads : omp_get_max_threads();
#endif
  /* one unit = `nh` query heads of one (sequence, kv_head) pair */
  const int nh = pairs >= threads ? group : 1;
  const long long units = pairs * (group / nh);
  a->units = (int32_t)units;
  a->threads_used = 1;
#ifdef _OPENMP
#pragma omp parallel num_threads(threads)
#endif
  {
#ifdef _OPENMP
#pragma omp single
    a->threads_used = omp_get_num_threads();
#endif
    float* qf = (float*)malloc(sizeof(float) * (size_t)group * d);
    float* krow = (float*)malloc(sizeof(float) * (size_t)d);
    float* acc = (float*)malloc(sizeof(float) * (size_t)group * d);
    float* scores = NULL;
    size_t scores_cap = 0;
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (long long u = 0; u < units; ++u) {
      const long long pr = u / (group / nh);
      const int h0 = (int)(u % (group / nh)) * nh;
      const int s = (int)(pr / hkv), kvh = (int)(pr % hkv);
      const int L = a->seq_lens[s];
      float* out = a->out + ((size_t)s * hq + (size_t)kvh * group + h0) * d;
      if (L <= 0) {
        memset(out, 0, sizeof(float) * (size_t)nh * d);
        continue;
      }
      if (scores_cap < (size_t)nh * L) {
        free(scores);
        scores_cap = (size_t)nh * L;
        scores = (float*)malloc(sizeof(float) * scores_cap);
      }
      if (!qf || !krow || !acc || !scores) {
        status = 2;
        continue;
      }
      for (int h = 0; h < nh; ++h) {
        const uint16_t* qr = q + s * a->q_stride_seq + (int64_t)(kvh * group + h0 + h) * a->q_stride_head;
        for (int i = 0; i < d; ++i) qf[h * d + i] = load16(qr + i, bf16) * a->scale;
      }
      const int32_t* bt = a->block_tables + (int64_t)s * a->bt_stride;
      for (int t = 0; t < L; ++t) {
        const int64_t pb = bt[t / bs];
        const uint16_t* kr = kc + pb * a->k_stride_block + (int64_t)(t % bs) * a->k_stride_token +
                             (int64_t)kvh * a->k_stride_head;
        for (int i = 0; i < d; ++i) krow[i] = load16(kr + i, bf16);
        for (int h = 0; h < nh; ++h) {
          float dot = 0.0f;
          for (int i = 0; i < d; ++i) dot += qf[h * d + i] * krow[i];
          scores[(size_t)h * L + t] = dot;
        }
      }
      for (int h = 0; h < nh; ++h) {
        float* sc = scores + (size_t)h * L;
        float m = -INFINITY;
        for (int t = 0; t < L; ++t) m = sc[t] > m ? sc[t] : m;
        float sum = 0.0f;
        for (int t = 0; t < L; ++t) {
          sc[t] = expf(sc[t] - m);
          sum += sc[t];
        }
        const float inv = 1.0f / sum;
        for (int t = 0; t < L; ++t) sc[t] *= inv;
      }
      memset(acc, 0, sizeof(float) * (size_t)nh * d);
      for (int t = 0; t < L; ++t) {
        const int64_t pb = bt[t / bs];
        const uint16_t* vr = vc + pb * a->v_stride_block + (int64_t)(t % bs) * a->v_stride_token +
                             (int64_t)kvh * a->v_stride_head;
        for (int i = 0; i < d; ++i) krow[i] = load16(vr + i, bf16);
        for (int h = 0; h < nh; ++h) {
          const float p = scores[(size_t)h * L + t];
          float* ac = acc + (size_t)h * d;
          for (int i = 0; i < d; ++i) ac[i] += p * krow[i];
        }
      }
      memcpy(out, acc, sizeof(float) * (size_t)nh * d);
    }
    free(qf);
    free(krow);
    free(acc);
    free(scores);
  }
  return status;
}

int dk_oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
