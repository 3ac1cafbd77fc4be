/* candidate_kernel for i8_matmul_bias_gelu_hmx backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, const int8_t *gelu_lut, int8_t *out, int n) {
    oracle_gemm_hmx_ex_rows(A, B, 0, out, n, n, n, 0, ORACLE_HMX_STORE_LUT_I8, ORACLE_HMX_ACT_NONE, bias, ORACLE_HMX_RES_NONE, NULL, gelu_lut, 0, 0, n);
}
