/* New task header for the u8 x s8 asymmetric GEMM with per-output-channel
 * requant to u8 (the M=16384, N=K=8192 benchmark case).  No corpus bundle has
 * this shape or epilogue; it composes four bundles' formulas:
 *   acc[i,j] = sum_k A[i*K+k] * B[k*N+j] - zpA * colsum[j]    (int32;
 *              gemm_tile_zp_i8/reference.c:10-19, colsum[j] = sum_k B[k*N+j])
 *   biased   = (int64) acc + bias[j]          (i8_gemm_bias_requant/reference.c:13)
 *   v        = biased * mult[j]                (requant_per_channel/reference.c:5-9,
 *                                               channel = output column j)
 *   r        = round_half_away(v >> shift[j]) + zp_out
 *   out      = clamp(r, 0, 255)                (requantize_i32_u8_dma/reference.c:5-13)
 * A [M,K] u8 row-major, B [K,N] s8 row-major, bias/mult/shift [N]. */
#ifndef HEXCUDA_KAPI_GEMM_U8S8_PC_H
#define HEXCUDA_KAPI_GEMM_U8S8_PC_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias,
                      uint8_t *out, int M, int N, int K, int32_t zpA,
                      const int32_t *mult, const int *shift, uint8_t zp_out);
#endif
