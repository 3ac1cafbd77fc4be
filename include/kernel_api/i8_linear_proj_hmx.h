/* candidate_kernel of kernels/expert/i8_linear_proj_hmx/kernel_api.h:25
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int8 saturated out, + bias[j], W is [out][in] (B transposed). */
#ifndef HEXCUDA_KAPI_I8_LINEAR_PROJ_HMX_H
#define HEXCUDA_KAPI_I8_LINEAR_PROJ_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *X, const int8_t *W, const int32_t *bias, int8_t *out, int n);
#endif
