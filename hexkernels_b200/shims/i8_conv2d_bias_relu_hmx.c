/* candidate_kernel for i8_conv2d_bias_relu_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_conv2d_bias_relu_hmx.h"
void candidate_kernel(const uint8_t *in, const int8_t *W, const int32_t *bias, int32_t *out, int n) {
    (void)n;
    hexcuda_host_conv2d_hmx(in, W, bias, out, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_RELU, 8, 10, 10, 32, 3, 3, 1);
}
