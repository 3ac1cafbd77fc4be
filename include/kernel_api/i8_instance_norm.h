/* candidate_kernel of kernels/expert/i8_instance_norm/kernel_api.h:29
 * int8 instance norm: per channel over H x W, per-channel gamma, beta and table. */
#ifndef HEXCUDA_KAPI_I8_INSTANCE_NORM_H
#define HEXCUDA_KAPI_I8_INSTANCE_NORM_H
#include <stdint.h>
void candidate_kernel(const int8_t *x, int8_t *out, int H, int W, int C, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut);
#endif
