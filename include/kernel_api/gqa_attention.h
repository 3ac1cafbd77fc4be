/* candidate_kernel of kernels/expert/gqa_attention/kernel_api.h:40
 * int8 GQA attention, requant scores, exp-table softmax, requant P.V. */
#ifndef HEXCUDA_KAPI_GQA_ATTENTION_H
#define HEXCUDA_KAPI_GQA_ATTENTION_H
#include <stdint.h>
/* the task's fixed shape */
#define H_Q 4
#define H_KV 2
#define GROUP_SIZE 2
#define SEQ 8
#define HEAD_DIM 16
void candidate_kernel(const int8_t *Q, const int8_t *K, const int8_t *V, const uint8_t *exp_lut,
                      int8_t *out, int32_t scale_mult, int scale_shift, int32_t av_mult, int av_shift);
#endif
