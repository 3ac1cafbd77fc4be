/* candidate_kernel of kernels/expert/i8_mean_dma/kernel_api.h:7
 * int8 mean: int32 sum / n, truncated. */
#ifndef HEXCUDA_KAPI_I8_MEAN_DMA_H
#define HEXCUDA_KAPI_I8_MEAN_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int32_t *out);
#endif
