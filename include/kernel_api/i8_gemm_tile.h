/* candidate_kernel of kernels/expert/i8_gemm_tile/kernel_api.h:5
 * s8 x s8 GEMM, B row-major [K,N], int32 out. */
#ifndef HEXCUDA_KAPI_I8_GEMM_TILE_H
#define HEXCUDA_KAPI_I8_GEMM_TILE_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K);
#endif
