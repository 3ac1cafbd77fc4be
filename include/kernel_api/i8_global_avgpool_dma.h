/* candidate_kernel of kernels/expert/i8_global_avgpool_dma/kernel_api.h:9
 * int8 mean (int32 sum / n, truncated) as int8. */
#ifndef HEXCUDA_KAPI_I8_GLOBAL_AVGPOOL_DMA_H
#define HEXCUDA_KAPI_I8_GLOBAL_AVGPOOL_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int8_t *out);
#endif
