/* candidate_kernel for fp16_attention_av_hmx on the B200: P . V, row-major V. */
#include "hexcuda.h"
#include "kernel_api/fp16_attention_av_hmx.h"
void candidate_kernel(const hvx_hf *P, const hvx_hf *V, hvx_hf *out, int n, int k_dim) {
    hexcuda_host_gemm_f16_nn((const uint16_t *)P, (const uint16_t *)V, (uint16_t *)out, n, n,
                             k_dim);
}
