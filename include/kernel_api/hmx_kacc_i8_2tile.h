/* candidate_kernel of kernels/expert/hmx_kacc_i8_2tile/kernel_api.h:14
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out. */
#ifndef HEXCUDA_KAPI_HMX_KACC_I8_2TILE_H
#define HEXCUDA_KAPI_HMX_KACC_I8_2TILE_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n, int K);
#endif
