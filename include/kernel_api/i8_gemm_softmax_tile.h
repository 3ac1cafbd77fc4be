/* candidate_kernel of kernels/expert/i8_gemm_softmax_tile/kernel_api.h:31
 * 16 x 16 x 16 int8 GEMM, sat8 scores, exp-table row softmax (the task's fixed GM = GN = GK = 16). */
#ifndef HEXCUDA_KAPI_I8_GEMM_SOFTMAX_TILE_H
#define HEXCUDA_KAPI_I8_GEMM_SOFTMAX_TILE_H
#include <stdint.h>
void candidate_kernel(const int8_t *A, const int8_t *B, uint8_t *out, const uint8_t *exp_lut);
#endif
