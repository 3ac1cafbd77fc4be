/* candidate_kernel of kernels/expert/matmul_residual_add_i8/kernel_api.h:22
 * s8 x s8 GEMM + requant, int8 residual added with saturation. */
#ifndef HEXCUDA_KAPI_MATMUL_RESIDUAL_ADD_I8_H
#define HEXCUDA_KAPI_MATMUL_RESIDUAL_ADD_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, const int8_t *residual, int8_t *out, int M, int N, int K, int32_t scale_mult, int scale_shift);
#endif
