/* candidate_kernel of kernels/expert/i8_gemm_gelu_lut/kernel_api.h:12
 * s8 x s8 GEMM, saturate, GELU table. */
#ifndef HEXCUDA_KAPI_I8_GEMM_GELU_LUT_H
#define HEXCUDA_KAPI_I8_GEMM_GELU_LUT_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, const int8_t *gelu_lut, int8_t *out, int M, int N, int K);
#endif
