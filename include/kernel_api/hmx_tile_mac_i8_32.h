/* candidate_kernel of kernels/expert/hmx_tile_mac_i8_32/kernel_api.h:13
 * u8 x s8 GEMM, v = sx12((acc * 17 + 8) >> 4); int32 out. */
#ifndef HEXCUDA_KAPI_HMX_TILE_MAC_I8_32_H
#define HEXCUDA_KAPI_HMX_TILE_MAC_I8_32_H
#include <stdint.h>
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n);
#endif
