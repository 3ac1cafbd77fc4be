/* candidate_kernel of kernels/expert/i8_decoder_block/kernel_api.h:53
 * int8 decoder block: causal exp-table attention, residual, LUT-activated FFN. */
#ifndef HEXCUDA_KAPI_I8_DECODER_BLOCK_H
#define HEXCUDA_KAPI_I8_DECODER_BLOCK_H
#include <stdint.h>
void candidate_kernel(const uint8_t *X,
                      const int8_t *W1, const int32_t *b1,
                      const int8_t *act_lut,
                      const int8_t *W2, const int32_t *b2,
                      const uint8_t *exp_lut,
                      int8_t *out, int S, int D, int Dff);
#endif
