/* candidate_kernel of kernels/expert/gemm_bias_gelu/kernel_api.h:14
 * s8 x s8 GEMM + bias (int64), saturate, GELU table. */
#ifndef HEXCUDA_KAPI_GEMM_BIAS_GELU_H
#define HEXCUDA_KAPI_GEMM_BIAS_GELU_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, const int8_t *gelu_lut, int8_t *out, int M, int N, int K);
#endif
