/* candidate_kernel of kernels/expert/hmx_matmul_i8_gelu_lut/kernel_api.h:12
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out = lut[v + 128]. */
#ifndef HEXCUDA_KAPI_HMX_MATMUL_I8_GELU_LUT_H
#define HEXCUDA_KAPI_HMX_MATMUL_I8_GELU_LUT_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *lut, int32_t *out, int n);
#endif
