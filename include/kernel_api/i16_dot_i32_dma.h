/* candidate_kernel of kernels/expert/i16_dot_i32_dma/kernel_api.h:8
 * int16 dot product, low 32 bits of the exact sum. */
#ifndef HEXCUDA_KAPI_I16_DOT_I32_DMA_H
#define HEXCUDA_KAPI_I16_DOT_I32_DMA_H
#include <stdint.h>
void candidate_kernel(const int16_t *a, const int16_t *b, int n, int32_t *out);
#endif
