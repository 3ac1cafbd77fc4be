/* candidate_kernel of kernels/expert/i8_mul_requant_dma/kernel_api.h:14
 * elementwise requant: pre mul_add, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_I8_MUL_REQUANT_DMA_H
#define HEXCUDA_KAPI_I8_MUL_REQUANT_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, const int8_t *b, int8_t *out, int n, int32_t mult, int shift, int8_t zp);
#endif
