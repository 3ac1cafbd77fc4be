/* candidate_kernel of kernels/expert/hmx_matmul_i8_bias_relu/kernel_api.h:13
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out, + bias[j], ReLU. */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_I8_BIAS_RELU_H
#define HEXCUDA_KAPI_HMX_MATMUL_I8_BIAS_RELU_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, int32_t *out, int n);
#endif
