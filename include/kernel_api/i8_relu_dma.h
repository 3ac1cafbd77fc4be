/* candidate_kernel of kernels/expert/i8_relu_dma/kernel_api.h:6
 * int8 ReLU. */
#ifndef HEXCUDA_KAPI_I8_RELU_DMA_H
#define HEXCUDA_KAPI_I8_RELU_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, int8_t *out, int n);
#endif
