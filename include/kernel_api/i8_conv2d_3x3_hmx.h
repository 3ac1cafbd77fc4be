/* candidate_kernel of kernels/expert/i8_conv2d_3x3_hmx/kernel_api.h:25
 * HMX-field 3x3 convolution, 8 -> 32 channels, 10 x 10 input (kernel_api.h:14-24); n (the output
 * positions) is not read. */
#ifndef HEXCUDA_KAPI_I8_CONV2D_3X3_HMX_H
#define HEXCUDA_KAPI_I8_CONV2D_3X3_HMX_H
#include <stdint.h>
void candidate_kernel(const uint8_t *in, const int8_t *W, uint16_t *out, int n);
#endif
