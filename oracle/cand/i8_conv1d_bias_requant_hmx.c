/* candidate_kernel for i8_conv1d_bias_requant_hmx backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const uint8_t *in, const int8_t *W, const int32_t *bias, int8_t *out, int n) {
    (void)n;
    oracle_conv2d_hmx(in, W, bias, out, ORACLE_HMX_STORE_I8_SAT, ORACLE_HMX_ACT_NONE, 16, 1, 68, 64, 1, 5, 1);
}
