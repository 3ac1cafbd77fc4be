/* candidate_kernel of kernels/expert/mlp_block/kernel_api.h:20
 * two-layer int8 MLP: GEMM + b1 + sat8 + GELU table, GEMM + b2 + requant. */
#ifndef HEXCUDA_KAPI_MLP_BLOCK_H
#define HEXCUDA_KAPI_MLP_BLOCK_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *W1, const int32_t *b1, const int8_t *gelu_lut, const int8_t *W2, const int32_t *b2, int8_t *out, int M, int K, int V, int D, int32_t mult, int shift, int8_t zp);
#endif
