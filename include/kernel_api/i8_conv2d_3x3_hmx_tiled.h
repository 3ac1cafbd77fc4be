/* candidate_kernel of kernels/expert/i8_conv2d_3x3_hmx_tiled/kernel_api.h:30
 * HMX-field 3x3 convolution, 8 -> 96 channels, 14 x 14 input (kernel_api.h:19-29); n (the output
 * positions) is not read. */
#ifndef HEXCUDA_KAPI_I8_CONV2D_3X3_HMX_TILED_H
#define HEXCUDA_KAPI_I8_CONV2D_3X3_HMX_TILED_H
#include <stdint.h>
void candidate_kernel(const uint8_t *in, const int8_t *W, uint16_t *out, int n);
#endif
