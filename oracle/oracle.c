/*
 * oracle.c — CPU restatement of the reference's GGUF dequant / MUL_MAT oracle.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library
 * and the timed CPU baseline.  It is never linked into, called by, or used as
 * a fallback for the product path (spiral_b200/libspiral_b200.so); only
 * tests/, __graft_entry__.smoke() and bench.py (cpu_baseline / reference arm)
 * load it.
 *
 * It restates, in C with OpenMP, the NumPy oracle of the reference:
 *   Q4_0  src/quants/tests/formats/q4_0.py:42-62   value = (q - 8) * d
 *   Q8_0  src/quants/tests/formats/q8_0.py:43-60   value = q * d
 *   Q6_K  src/quants/tests/formats/q6_k.py:55-112  value = d * sc * (q - 32)
 * followed by ml_dtypes' float32 -> bfloat16 cast (round to nearest even;
 * NaN keeps its sign and gets the quiet bit), and the fp32 matmul of
 * src/quants/tests/mmul.py:104-112.  Output layout is ggml row-major [N][K]
 * (the reference's reference_weights order [N/8][K][8] is a re-tiling of it).
 *
 * Pinning: tests/test_oracle.py checks this file bit for bit against golden
 * vectors produced by the reference's own Python oracle
 * (tests/golden/make_golden.py) and against SHA-256 digests of its outputs at
 * the full BASELINE sizes.
 */
#include "oracle.h"

#include <math.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

int64_t oracle_block_k(int fmt) {
  return fmt == ORACLE_Q4_0 ? 32 : fmt == ORACLE_Q8_0 ? 32 : fmt == ORACLE_Q6_K ? 256 : 0;
}

int64_t oracle_block_bytes(int fmt) {
  return fmt == ORACLE_Q4_0 ? 18 : fmt == ORACLE_Q8_0 ? 34 : fmt == ORACLE_Q6_K ? 210 : 0;
}

/* IEEE binary16 -> binary32, exact (np.float16(...).astype(np.float32)).
 * ftz: subnormal values (exponent 0, mantissa != 0) become +0, as the
 * reference repack stores them (src/quants/common/repack.h:29-34,
 * q4_0/repack.h:75-80); signed zeros are kept. */
float oracle_fp16_to_f32(uint16_t h, int ftz) {
  const int sign = (h >> 15) & 1;
  const int exp = (h >> 10) & 0x1f;
  const int mant = h & 0x3ff;
  float v;
  if (exp == 0) {
    if (ftz && mant != 0) return 0.0f;
    v = ldexpf((float)mant, -24);
  } else if (exp == 31) {
    v = mant ? NAN : INFINITY;
  } else {
    v = ldexpf((float)(mant | 0x400), exp - 25);
  }
  return sign ? -v : v;
}

/* float32 -> bfloat16 bits, round to nearest even (ml_dtypes semantics). */
uint16_t oracle_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof(u));
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float bf16_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, sizeof(f));
  return f;
}

static inline uint16_t ld16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* One canonical block -> block_k float values (exact products). */
static void dequant_block(int fmt, const uint8_t* b, float* y, int ftz) {
  if (fmt == ORACLE_Q4_0) {
    /* q4_0.py:52-60 */
    const float d = oracle_fp16_to_f32(ld16(b), ftz);
    for (int j = 0; j < 16; ++j) {
      y[j] = ((float)(b[2 + j] & 0x0f) - 8.0f) * d;
      y[j + 16] = ((float)(b[2 + j] >> 4) - 8.0f) * d;
    }
  } else if (fmt == ORACLE_Q8_0) {
    /* q8_0.py:50-58 */
    const float d = oracle_fp16_to_f32(ld16(b), ftz);
    for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)b[2 + j] * d;
  } else {
    /* q6_k.py:55-97 */
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    const float d = oracle_fp16_to_f32(ld16(b + 208), ftz);
    for (int h = 0; h < 2; ++h) {
      for (int l = 0; l < 32; ++l) {
        const int is = l / 16;
        const int qhb = qh[32 * h + l];
        const int q1 = ((ql[64 * h + l] & 0x0f) | (((qhb >> 0) & 3) << 4)) - 32;
        const int q2 = ((ql[64 * h + 32 + l] & 0x0f) | (((qhb >> 2) & 3) << 4)) - 32;
        const int q3 = ((ql[64 * h + l] >> 4) | (((qhb >> 4) & 3) << 4)) - 32;
        const int q4 = ((ql[64 * h + 32 + l] >> 4) | (((qhb >> 6) & 3) << 4)) - 32;
        /* (d * sc) * q, in that order, as the reference evaluates it: every
         * product is exact in float (<= 24 significant bits) and the order
         * fixes the sign of a zero result (q == 32 or sc == 0). */
        y[128 * h + l] = (d * (float)sc[8 * h + is]) * (float)q1;
        y[128 * h + 32 + l] = (d * (float)sc[8 * h + is + 2]) * (float)q2;
        y[128 * h + 64 + l] = (d * (float)sc[8 * h + is + 4]) * (float)q3;
        y[128 * h + 96 + l] = (d * (float)sc[8 * h + is + 6]) * (float)q4;
      }
    }
  }
}

static void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

/* Threads an OpenMP region started now would use (after set_threads), so a
 * timed CPU baseline can report the cores it really ran on: torchrun sets
 * OMP_NUM_THREADS=1 in every rank, which the default would silently take. */
int oracle_threads(int threads) {
  set_threads(threads);
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_dequant_f32(int fmt, const uint8_t* src, int64_t src_stride, float* out, int64_t K, int64_t N, int ftz,
                        int threads) {
  const int64_t bk = oracle_block_k(fmt), bb = oracle_block_bytes(fmt);
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t b = 0; b < K / bk; ++b) dequant_block(fmt, src + n * src_stride + b * bb, out + n * K + b * bk, ftz);
  }
}

void oracle_dequant_bf16(int fmt, const uint8_t* src, int64_t src_stride, uint16_t* out, int64_t K, int64_t N,
                         int ftz, int threads) {
  const int64_t bk = oracle_block_k(fmt), bb = oracle_block_bytes(fmt);
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    float y[256];
    for (int64_t b = 0; b < K / bk; ++b) {
      dequant_block(fmt, src + n * src_stride + b * bb, y, ftz);
      for (int64_t j = 0; j < bk; ++j) out[n * K + b * bk + j] = oracle_f32_to_bf16(y[j]);
    }
  }
}

/* y[m][n] = sum_k bf16(W[n][k]) * x[m][k], accumulated in double: the
 * high-precision reference the tolerance tests compare against. */
void oracle_mul_mat_f64(int fmt, const uint8_t* w, int64_t w_stride, const uint16_t* x, int64_t x_stride, double* y,
                        int64_t M, int64_t N, int64_t K, int ftz, int threads) {
  const int64_t bk = oracle_block_k(fmt), bb = oracle_block_bytes(fmt);
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    float blk[256];
    double acc[64];
    const int64_t mm = M < 64 ? M : 64;
    for (int64_t m0 = 0; m0 < M; m0 += mm) {
      const int64_t mc = (M - m0) < mm ? (M - m0) : mm;
      for (int64_t m = 0; m < mc; ++m) acc[m] = 0.0;
      for (int64_t b = 0; b < K / bk; ++b) {
        dequant_block(fmt, w + n * w_stride + b * bb, blk, ftz);
        for (int64_t j = 0; j < bk; ++j) {
          const double wv = (double)bf16_to_f32(oracle_f32_to_bf16(blk[j]));
          const int64_t k = b * bk + j;
          for (int64_t m = 0; m < mc; ++m) acc[m] += wv * (double)bf16_to_f32(x[(m0 + m) * x_stride + k]);
        }
      }
      for (int64_t m = 0; m < mc; ++m) y[(m0 + m) * N + n] = acc[m];
    }
  }
}

/* The reference's CPU path as a timed baseline: dequantize each weight row to
 * bf16, widen to fp32, and accumulate the dot products in fp32
 * (mmul.py:104-112 "inputs_rows @ weights_matrix" with fp32 operands). */
void oracle_mul_mat_f32(int fmt, const uint8_t* w, int64_t w_stride, const uint16_t* x, int64_t x_stride, float* y,
                        int64_t M, int64_t N, int64_t K, int ftz, int threads) {
  const int64_t bk = oracle_block_k(fmt), bb = oracle_block_bytes(fmt);
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    float blk[256];
    float acc[64];
    const int64_t mm = M < 64 ? M : 64;
    for (int64_t m0 = 0; m0 < M; m0 += mm) {
      const int64_t mc = (M - m0) < mm ? (M - m0) : mm;
      for (int64_t m = 0; m < mc; ++m) acc[m] = 0.0f;
      for (int64_t b = 0; b < K / bk; ++b) {
        dequant_block(fmt, w + n * w_stride + b * bb, blk, ftz);
        for (int64_t j = 0; j < bk; ++j) blk[j] = bf16_to_f32(oracle_f32_to_bf16(blk[j]));
        for (int64_t m = 0; m < mc; ++m) {
          const uint16_t* xr = x + (m0 + m) * x_stride + b * bk;
          float s = 0.0f;
          for (int64_t j = 0; j < bk; ++j) s += blk[j] * bf16_to_f32(xr[j]);
          acc[m] += s;
        }
      }
      for (int64_t m = 0; m < mc; ++m) y[(m0 + m) * N + n] = acc[m];
    }
  }
}
