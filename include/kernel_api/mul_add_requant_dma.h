/* candidate_kernel of kernels/expert/mul_add_requant_dma/kernel_api.h:18
 * elementwise requant: pre mul_add, round half away, clamp, int8 out. */
#ifndef HEXCUDA_KAPI_MUL_ADD_REQUANT_DMA_H
#define HEXCUDA_KAPI_MUL_ADD_REQUANT_DMA_H
#include <stdint.h>
void candidate_kernel(const int32_t *a, const int32_t *b, int8_t *out, int n);
#endif
