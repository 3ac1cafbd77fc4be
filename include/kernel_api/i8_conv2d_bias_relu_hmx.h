/* candidate_kernel of kernels/expert/i8_conv2d_bias_relu_hmx/kernel_api.h:23
 * HMX-field 3x3 convolution + bias + ReLU, int32 out (kernel_api.h:12-22); n (the output
 * positions) is not read. */
#ifndef HEXCUDA_KAPI_I8_CONV2D_BIAS_RELU_HMX_H
#define HEXCUDA_KAPI_I8_CONV2D_BIAS_RELU_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *in, const int8_t *W, const int32_t *bias, int32_t *out, int n);
#endif
