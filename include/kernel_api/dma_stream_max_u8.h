/* candidate_kernel of kernels/expert/dma_stream_max_u8/kernel_api.h:12
 * maximum of a uint8 array (0 for n = 0). */
#ifndef HEXCUDA_KAPI_DMA_STREAM_MAX_U8_H
#define HEXCUDA_KAPI_DMA_STREAM_MAX_U8_H
#include <stdint.h>
void candidate_kernel(const uint8_t *a, int n, uint8_t *out);
#endif
