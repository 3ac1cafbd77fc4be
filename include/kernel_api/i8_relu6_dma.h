/* candidate_kernel of kernels/expert/i8_relu6_dma/kernel_api.h:9
 * int8 ReLU capped at (int8)(6 scale). */
#ifndef HEXCUDA_KAPI_I8_RELU6_DMA_H
#define HEXCUDA_KAPI_I8_RELU6_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, int8_t *out, int n, int8_t scale);
#endif
