/* candidate_kernel of kernels/expert/dma_double_buffer_relu_u8/kernel_api.h:11
 * uint8 max(a - 128, 0). */
#ifndef HEXCUDA_KAPI_DMA_DOUBLE_BUFFER_RELU_U8_H
#define HEXCUDA_KAPI_DMA_DOUBLE_BUFFER_RELU_U8_H
#include <stdint.h>
void candidate_kernel(const uint8_t *a, uint8_t *out, int n);
#endif
