/* candidate_kernel of kernels/expert/i8_ffn_block/kernel_api.h:29
 * HMX-convention two-layer int8 FFN (ReLU + shift 8 between, shift 3 after). */
#ifndef HEXCUDA_KAPI_I8_FFN_BLOCK_H
#define HEXCUDA_KAPI_I8_FFN_BLOCK_H
#include <stdint.h>
void candidate_kernel(const uint8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2, const int32_t *b2, int8_t *out, int S, int D, int Dff);
#endif
