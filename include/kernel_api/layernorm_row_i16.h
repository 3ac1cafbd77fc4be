/* candidate_kernel of kernels/expert/layernorm_row_i16/kernel_api.h:32
 * int16 row layernorm, per-column gamma / beta. */
#ifndef HEXCUDA_KAPI_LAYERNORM_ROW_I16_H
#define HEXCUDA_KAPI_LAYERNORM_ROW_I16_H
#include <stdint.h>
void candidate_kernel(const int16_t *x, int16_t *out, int R, int C, const int16_t *gamma, const int16_t *beta, const uint16_t *inv_lut);
#endif
