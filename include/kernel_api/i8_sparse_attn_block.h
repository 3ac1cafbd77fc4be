/* candidate_kernel of kernels/expert/i8_sparse_attn_block/kernel_api.h:36
 * int8 LUT-softmax attention with a banded (|i - j| <= window) score mask,
 * requant scores and output; fixed H 1, SEQ 8, HEAD_DIM 16 (kernel_api.h:32-34). */
#ifndef HEXCUDA_KAPI_I8_SPARSE_ATTN_BLOCK_H
#define HEXCUDA_KAPI_I8_SPARSE_ATTN_BLOCK_H
#include <stdint.h>
#define SPARSE_ATTN_H 1
#define SPARSE_ATTN_SEQ 8
#define SPARSE_ATTN_HEAD_DIM 16
void candidate_kernel(const int8_t *Q, const int8_t *K, const int8_t *V, const uint8_t *exp_lut, int8_t *out, int window, int32_t smult, int sshift, int32_t amult, int ashift);
#endif
