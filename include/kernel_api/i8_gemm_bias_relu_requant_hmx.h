/* candidate_kernel of kernels/expert/i8_gemm_bias_relu_requant_hmx/kernel_api.h:16-17
 * out uint8 = clamp(max(sx12((acc * 17 + 8) >> 4) + bias[j], 0), 0, 255). */
#ifndef HEXCUDA_KAPI_I8_GEMM_BIAS_RELU_REQUANT_HMX_H
#define HEXCUDA_KAPI_I8_GEMM_BIAS_RELU_REQUANT_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias,
                      uint8_t *out, int n);
#endif
