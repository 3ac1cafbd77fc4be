/* candidate_kernel of kernels/expert/i8_absmax_dma/kernel_api.h:7
 * absolute maximum of int8 (|-128| = 128). */
#ifndef HEXCUDA_KAPI_I8_ABSMAX_DMA_H
#define HEXCUDA_KAPI_I8_ABSMAX_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int n, int32_t *out);
#endif
