/* candidate_kernel of kernels/expert/gemm_tile_bias_relu_i8/kernel_api.h:17
 * s8 x s8 GEMM (Bt) + bias, ReLU, saturate to int8. */
#ifndef HEXCUDA_KAPI_GEMM_TILE_BIAS_RELU_I8_H
#define HEXCUDA_KAPI_GEMM_TILE_BIAS_RELU_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int8_t *C, int M, int N, int K);
#endif
