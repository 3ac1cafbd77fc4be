/* candidate_kernel of kernels/expert/i8_sign_dma/kernel_api.h:8
 * int8 sign (-1, 0, 1). */
#ifndef HEXCUDA_KAPI_I8_SIGN_DMA_H
#define HEXCUDA_KAPI_I8_SIGN_DMA_H
#include <stdint.h>
void candidate_kernel(const int8_t *in, int8_t *out, int n);
#endif
