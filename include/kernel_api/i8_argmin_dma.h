/* candidate_kernel of kernels/expert/i8_argmin_dma/kernel_api.h:8
 * first index of the int8 minimum. */
#ifndef HEXCUDA_KAPI_I8_ARGMIN_DMA_H
#define HEXCUDA_KAPI_I8_ARGMIN_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int32_t *out);
#endif
