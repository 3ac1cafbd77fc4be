/* candidate_kernel of kernels/expert/layernorm_residual/kernel_api.h:24
 * saturating residual add, then int8 layernorm of the one row. */
#ifndef HEXCUDA_KAPI_LAYERNORM_RESIDUAL_H
#define HEXCUDA_KAPI_LAYERNORM_RESIDUAL_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, const int8_t *residual, int8_t *out, int n, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut);
#endif
