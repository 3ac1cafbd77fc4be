/* candidate_kernel for fp16_attention_qkt_hmx on the B200: the n x n x k_dim
 * fp16 GEMM with K stored [n, k_dim] (column-major B). */
#include "hexcuda.h"
#include "kernel_api/fp16_attention_qkt_hmx.h"
void candidate_kernel(const hvx_hf *Q, const hvx_hf *K, hvx_hf *out, int n, int k_dim) {
    hexcuda_host_gemm_f16_nt((const uint16_t *)Q, (const uint16_t *)K, (uint16_t *)out, n, n,
                             k_dim);
}
