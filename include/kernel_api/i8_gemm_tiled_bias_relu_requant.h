/* candidate_kernel of kernels/expert/i8_gemm_tiled_bias_relu_requant/kernel_api.h:23
 * HMX field + bias, ReLU, saturate to u8. */
#ifndef HEXCUDA_KAPI_I8_GEMM_TILED_BIAS_RELU_REQUANT_H
#define HEXCUDA_KAPI_I8_GEMM_TILED_BIAS_RELU_REQUANT_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, uint8_t *out, int M, int N, int K);
#endif
