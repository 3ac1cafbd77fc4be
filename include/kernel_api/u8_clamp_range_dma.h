/* candidate_kernel of kernels/expert/u8_clamp_range_dma/kernel_api.h:8
 * uint8 clamp to [64, 191]. */
#ifndef HEXCUDA_KAPI_U8_CLAMP_RANGE_DMA_H
#define HEXCUDA_KAPI_U8_CLAMP_RANGE_DMA_H
#include <stdint.h>
void candidate_kernel(const uint8_t *in, uint8_t *out, int n);
#endif
