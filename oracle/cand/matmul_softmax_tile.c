/* candidate_kernel for matmul_softmax_tile backed by the oracle. */
#include <stddef.h>
#include <stdlib.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, uint8_t *out, const uint8_t *exp_lut, int32_t inv_sqrt_d, int shift) {
    int8_t sc[256];
    oracle_gemm_i8_rq_ex_rows(Q, K, 1, NULL, NULL, sc, 16, 16, 32, inv_sqrt_d, shift, 0, 0, 0, 16);
    oracle_lut_softmax_u8(sc, out, 16, 16, exp_lut, NULL);
}
