/* candidate_kernel of kernels/expert/u8_max_dma/kernel_api.h:7
 * maximum of a uint8 array (0 when empty). */
#ifndef HEXCUDA_KAPI_U8_MAX_DMA_H
#define HEXCUDA_KAPI_U8_MAX_DMA_H
#include <stdint.h>
void candidate_kernel(const uint8_t *a, int n, uint8_t *out);
#endif
