/* candidate_kernel of kernels/expert/i8_min_scalar_dma/kernel_api.h:8
 * elementwise min with a runtime int8 scalar. */
#ifndef HEXCUDA_KAPI_I8_MIN_SCALAR_DMA_H
#define HEXCUDA_KAPI_I8_MIN_SCALAR_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *in, int8_t *out, int n, int8_t c);
#endif
