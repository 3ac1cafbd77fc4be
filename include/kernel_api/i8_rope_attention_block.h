/* candidate_kernel of kernels/expert/i8_rope_attention_block/kernel_api.h:40
 * i8_attention_block after an int8 rotary rotation of Q and K. */
#ifndef HEXCUDA_KAPI_I8_ROPE_ATTENTION_BLOCK_H
#define HEXCUDA_KAPI_I8_ROPE_ATTENTION_BLOCK_H
#include <stdint.h>
void candidate_kernel(const uint8_t *Q, const int8_t *K, const int8_t *V,
                      const int8_t *cos_lut, const int8_t *sin_lut,
                      uint16_t *out, int S, int D, int rot_shift,
                      const uint8_t *exp_lut);
#endif
