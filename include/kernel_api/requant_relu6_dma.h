/* candidate_kernel of kernels/expert/requant_relu6_dma/kernel_api.h:15
 * elementwise requant: pre a, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_REQUANT_RELU6_DMA_H
#define HEXCUDA_KAPI_REQUANT_RELU6_DMA_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, int8_t *out, int n);
#endif
