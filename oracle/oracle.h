/*
 * oracle.h — CPU restatement of the reference's dequant / MUL_MAT oracle.
 * TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline); see oracle.c.
 */
#ifndef SPIRAL_ORACLE_H
#define SPIRAL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_Q4_0 = 2, ORACLE_Q8_0 = 8, ORACLE_Q6_K = 14 };

int64_t oracle_block_k(int fmt);
int64_t oracle_block_bytes(int fmt);
float oracle_fp16_to_f32(uint16_t h, int ftz);
uint16_t oracle_f32_to_bf16(float f);
/* Sets the OpenMP thread count when threads > 0; returns the count in effect. */
int oracle_threads(int threads);

/* out[n*K + k] = W[n][k]; src row n at src + n*src_stride. */
void oracle_dequant_f32(int fmt, const uint8_t* src, int64_t src_stride, float* out, int64_t K, int64_t N, int ftz,
                        int threads);
void oracle_dequant_bf16(int fmt, const uint8_t* src, int64_t src_stride, uint16_t* out, int64_t K, int64_t N,
                         int ftz, int threads);

/* y[m*N + n] = sum_k bf16(W[n][k]) * x[m*x_stride + k]. */
void oracle_mul_mat_f64(int fmt, const uint8_t* w, int64_t w_stride, const uint16_t* x, int64_t x_stride, double* y,
                        int64_t M, int64_t N, int64_t K, int ftz, int threads);
void oracle_mul_mat_f32(int fmt, const uint8_t* w, int64_t w_stride, const uint16_t* x, int64_t x_stride, float* y,
                        int64_t M, int64_t N, int64_t K, int ftz, int threads);

#ifdef __cplusplus
}
#endif

#endif
