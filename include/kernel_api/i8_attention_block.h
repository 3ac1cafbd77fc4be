/* candidate_kernel of kernels/expert/i8_attention_block/kernel_api.h:30
 * HMX-field scores, exp-table softmax, HMX field of P.V (uint16). */
#ifndef HEXCUDA_KAPI_I8_ATTENTION_BLOCK_H
#define HEXCUDA_KAPI_I8_ATTENTION_BLOCK_H
#include <stdint.h>
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V,
                      uint16_t *out, int S, int D, const uint8_t *exp_lut);
#endif
