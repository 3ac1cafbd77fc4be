/* candidate_kernel of kernels/expert/i8_conv1d_bias_requant_hmx/kernel_api.h:22
 * HMX-field 1-D convolution (width 5, 16 -> 64 channels, length 68) + bias, int8 saturation (kernel_api.h:15-21); n (the output
 * positions) is not read. */
#ifndef HEXCUDA_KAPI_I8_CONV1D_BIAS_REQUANT_HMX_H
#define HEXCUDA_KAPI_I8_CONV1D_BIAS_REQUANT_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *in, const int8_t *W, const int32_t *bias, int8_t *out, int n);
#endif
