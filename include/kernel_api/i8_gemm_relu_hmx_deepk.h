/* candidate_kernel of kernels/expert/i8_gemm_relu_hmx_deepk/kernel_api.h:15
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out, ReLU. */
#ifndef HEXCUDA_KAPI_I8_GEMM_RELU_HMX_DEEPK_H
#define HEXCUDA_KAPI_I8_GEMM_RELU_HMX_DEEPK_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n, int K);
#endif
