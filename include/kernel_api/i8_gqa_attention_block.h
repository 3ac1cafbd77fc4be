/* candidate_kernel of kernels/expert/i8_gqa_attention_block/kernel_api.h:40
 * GQA form of i8_attention_block at its fixed shape. */
#ifndef HEXCUDA_KAPI_I8_GQA_ATTENTION_BLOCK_H
#define HEXCUDA_KAPI_I8_GQA_ATTENTION_BLOCK_H
#include <stdint.h>
/* the task's fixed shape */
#define GQA_H_Q 2
#define GQA_H_KV 1
#define GQA_GROUP_SIZE 2
#define GQA_S 64
#define GQA_D 64
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V,
                      uint16_t *out, const uint8_t *exp_lut);
#endif
