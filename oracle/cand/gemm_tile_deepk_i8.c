/* candidate_kernel for gemm_tile_deepk_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K) {
    oracle_gemm_i8_acc_rows(A, 1, B, 0, NULL, NULL, 0, NULL, C, ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_NONE, M, N, K, 0, M);
}
