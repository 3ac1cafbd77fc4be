/* candidate_kernel of kernels/expert/i8_sum_dma/kernel_api.h:7
 * whole-array int8 sum, int32 accumulator. */
#ifndef HEXCUDA_KAPI_I8_SUM_DMA_H
#define HEXCUDA_KAPI_I8_SUM_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int32_t *out);
#endif
