/* candidate_kernel of kernels/expert/i8_matmul_bias_hmx/kernel_api.h:14
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out, + bias[j]. */
#ifndef HEXCUDA_KAPI_I8_MATMUL_BIAS_HMX_H
#define HEXCUDA_KAPI_I8_MATMUL_BIAS_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, int32_t *out, int n);
#endif
