/* candidate_kernel of kernels/expert/u8_global_avgpool_dma/kernel_api.h:9
 * uint8 mean (int32 sum / n, truncated) as uint8. */
#ifndef HEXCUDA_KAPI_U8_GLOBAL_AVGPOOL_DMA_H
#define HEXCUDA_KAPI_U8_GLOBAL_AVGPOOL_DMA_H
#include <stdint.h>
void candidate_kernel(const uint8_t *a, int n, uint8_t *out);
#endif
