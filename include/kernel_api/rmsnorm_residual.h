/* candidate_kernel of kernels/expert/rmsnorm_residual/kernel_api.h:23
 * saturating residual add, int8 RMS norm with an inverse table. */
#ifndef HEXCUDA_KAPI_RMSNORM_RESIDUAL_H
#define HEXCUDA_KAPI_RMSNORM_RESIDUAL_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, const int8_t *residual, int8_t *out, int n, const int8_t *gamma, const uint8_t *inv_lut);
#endif
