/* candidate_kernel for fp16_matmul_residual on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/fp16_matmul_residual.h"
#define U(p) ((const uint16_t *)(p))
#define W(p) ((uint16_t *)(p))
void candidate_kernel(const hvx_hf *A, const hvx_hf *B, const hvx_hf *C, hvx_hf *out, int n, int k_dim) {
    hexcuda_host_gemm_f16_ex(U(A), U(B), 0, NULL, U(C), W(out), HEXCUDA_F16_ACT_NONE, HEXCUDA_F16_PREROUND_ACC, 1.0f, n, n, k_dim);
}
