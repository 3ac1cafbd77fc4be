/* candidate_kernel for gelu_ffn_residual backed by the oracle. */
#include <stddef.h>
#include <stdlib.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *x, const int8_t *W1, const int32_t *b1, const int8_t *gelu_lut, const int8_t *W2, const int32_t *b2, const int8_t *x_res, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut, int8_t *out, int M, int K, int V, int D) {
    int8_t *hid = (int8_t *)malloc((size_t)M * V), *s = (int8_t *)malloc((size_t)M * D);
    oracle_gemm_i8_acc_rows(x, 1, W1, 0, b1, NULL, 0, gelu_lut, hid, ORACLE_HMX_STORE_LUT_I8, ORACLE_HMX_ACT_NONE, M, V, K, 0, M);
    oracle_gemm_i8_acc_rows(hid, 1, W2, 0, b2, x_res, ORACLE_HMX_RES_I8, NULL, s, ORACLE_HMX_STORE_I8_SAT, ORACLE_HMX_ACT_NONE, M, D, V, 0, M);
    oracle_layernorm_lut_i8(s, NULL, NULL, out, M, D, gamma, beta, inv_lut, 0);
    free(hid);
    free(s);
}
