/* candidate_kernel of kernels/expert/matmul_softmax_tile/kernel_api.h:33
 * 16 x 16 Q K^T (head dim 32) requantised to int8, exp-table row softmax (the task's fixed SEQ_Q = SEQ_K = 16, HEAD_DIM = 32). */
#ifndef HEXCUDA_KAPI_MATMUL_SOFTMAX_TILE_H
#define HEXCUDA_KAPI_MATMUL_SOFTMAX_TILE_H
#include <stdint.h>
void candidate_kernel(const int8_t *Q, const int8_t *K, uint8_t *out, const uint8_t *exp_lut, int32_t inv_sqrt_d, int shift);
#endif
