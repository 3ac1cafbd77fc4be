/* candidate_kernel of kernels/expert/i8_matmul_bias_gelu_hmx/kernel_api.h:16
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int8 out = gelu_lut[sat_i8(v) + 128], + bias[j]. */
#ifndef HEXCUDA_KAPI_I8_MATMUL_BIAS_GELU_HMX_H
#define HEXCUDA_KAPI_I8_MATMUL_BIAS_GELU_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, const int8_t *gelu_lut, int8_t *out, int n);
#endif
