/* candidate_kernel of kernels/expert/requantize_i32_i8_dma/kernel_api.h:13
 * elementwise requant: pre a, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_REQUANTIZE_I32_I8_DMA_H
#define HEXCUDA_KAPI_REQUANTIZE_I32_I8_DMA_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, int8_t *out, int n, int32_t mult, int shift, int8_t zp);
#endif
