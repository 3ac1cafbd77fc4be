/* candidate_kernel of kernels/expert/i8_vadd_dma/kernel_api.h:7
 * int8 wrapping add (the low byte of the sum). */
#ifndef HEXCUDA_KAPI_I8_VADD_DMA_H
#define HEXCUDA_KAPI_I8_VADD_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *b, int8_t *out, int n);
#endif
