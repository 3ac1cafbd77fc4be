/* candidate_kernel of kernels/expert/u8_threshold_dma/kernel_api.h:8
 * uint8 threshold: 255 where in >= 128, else 0. */
#ifndef HEXCUDA_KAPI_U8_THRESHOLD_DMA_H
#define HEXCUDA_KAPI_U8_THRESHOLD_DMA_H
#include <stdint.h>
void candidate_kernel(const uint8_t *in, uint8_t *out, int n);
#endif
