/* candidate_kernel for hmx_matmul_fp16_deepk (kernel_api.h:10) backed by the oracle:
 * an n x n x k_dim GEMM with row-major B[k_dim][n]. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n, int k_dim) {
    oracle_gemm_f16_nn_rows((const uint16_t *)A, (const uint16_t *)B, (uint16_t *)out,
                            n, n, k_dim, 0, n);
}
