/* candidate_kernel of kernels/expert/i8_global_maxpool_dma/kernel_api.h:8
 * int8 maximum (-128 when empty). */
#ifndef HEXCUDA_KAPI_I8_GLOBAL_MAXPOOL_DMA_H
#define HEXCUDA_KAPI_I8_GLOBAL_MAXPOOL_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int8_t *out);
#endif
