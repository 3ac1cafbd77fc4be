/* candidate_kernel of kernels/expert/gqa_group_reduce_i8/kernel_api.h:38
 * head-group reduce: sum of each group's H/G head planes, requant to int8. */
#ifndef HEXCUDA_KAPI_GQA_GROUP_REDUCE_I8_H
#define HEXCUDA_KAPI_GQA_GROUP_REDUCE_I8_H
#include <stdint.h>
void candidate_kernel(const int8_t *X, int8_t *Y, int H, int G, int M, int N, int32_t scale_mult, int scale_shift);
#endif
