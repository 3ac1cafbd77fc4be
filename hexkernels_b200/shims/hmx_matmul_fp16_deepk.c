/* candidate_kernel for hmx_matmul_fp16_deepk on the B200: row-major-B fp16 GEMM. */
#include "hexcuda.h"
#include "kernel_api/hmx_matmul_fp16_deepk.h"
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, hvx_hf *out, int n, int k_dim) {
    hexcuda_host_gemm_f16_nn((const uint16_t *)A, (const uint16_t *)B, (uint16_t *)out, n, n,
                             k_dim);
}
