/* candidate_kernel of kernels/expert/i8_dot_i32_dma/kernel_api.h:8
 * int8 dot product, int32 out. */
#ifndef HEXCUDA_KAPI_I8_DOT_I32_DMA_H
#define HEXCUDA_KAPI_I8_DOT_I32_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *b, int n, int32_t *out);
#endif
