/* candidate_kernel of kernels/expert/requant_add_dma/kernel_api.h:16
 * elementwise requant: pre add, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_REQUANT_ADD_DMA_H
#define HEXCUDA_KAPI_REQUANT_ADD_DMA_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n);
#endif
