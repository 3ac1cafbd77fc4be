/* candidate_kernel for i8_conv2d_bias_relu_hmx backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const uint8_t *in, const int8_t *W, const int32_t *bias, int32_t *out, int n) {
    (void)n;
    oracle_conv2d_hmx(in, W, bias, out, ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_RELU, 8, 10, 10, 32, 3, 3, 1);
}
