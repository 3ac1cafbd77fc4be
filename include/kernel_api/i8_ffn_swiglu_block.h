/* candidate_kernel of kernels/expert/i8_ffn_swiglu_block/kernel_api.h:45
 * HMX-convention int8 SwiGLU FFN (shifts 2 / 2, gate shift 10, zero point 8, output shift 3). */
#ifndef HEXCUDA_KAPI_I8_FFN_SWIGLU_BLOCK_H
#define HEXCUDA_KAPI_I8_FFN_SWIGLU_BLOCK_H
#include <stdint.h>
void candidate_kernel(const uint8_t *X, const int8_t *Wg, const int8_t *Wu, const int8_t *Wd, const int32_t *bd, const uint8_t *silu_lut, int8_t *out, int S, int D, int Dff);
#endif
