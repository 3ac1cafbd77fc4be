/* candidate_kernel of kernels/expert/i8_top1_reduce_dma/kernel_api.h:9
 * int8 maximum and its first index. */
#ifndef HEXCUDA_KAPI_I8_TOP1_REDUCE_DMA_H
#define HEXCUDA_KAPI_I8_TOP1_REDUCE_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int32_t *out);
#endif
