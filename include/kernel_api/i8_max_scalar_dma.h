/* candidate_kernel of kernels/expert/i8_max_scalar_dma/kernel_api.h:7
 * elementwise max with a runtime int8 scalar. */
#ifndef HEXCUDA_KAPI_I8_MAX_SCALAR_DMA_H
#define HEXCUDA_KAPI_I8_MAX_SCALAR_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *in, int8_t *out, int n, int8_t c);
#endif
