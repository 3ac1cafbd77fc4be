/* candidate_kernel of kernels/expert/hmx_gemv_i8/kernel_api.h:10
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out. */
#ifndef HEXCUDA_KAPI_HMX_GEMV_I8_H
#define HEXCUDA_KAPI_HMX_GEMV_I8_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *x, int32_t *out, int n);
#endif
