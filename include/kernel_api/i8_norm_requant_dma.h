/* candidate_kernel of kernels/expert/i8_norm_requant_dma/kernel_api.h:18
 * 16-channel normalisation requant then requant (5, 4, 0); the task's tables. */
#ifndef HEXCUDA_KAPI_I8_NORM_REQUANT_DMA_H
#define HEXCUDA_KAPI_I8_NORM_REQUANT_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *a, int8_t *out, int n);
#endif
