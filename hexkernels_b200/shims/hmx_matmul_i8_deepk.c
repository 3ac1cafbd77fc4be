/* candidate_kernel for hmx_matmul_i8_deepk on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/hmx_matmul_i8_deepk.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, int32_t *out, int n, int K) {
    hexcuda_host_gemm_hmx(A, B, 0, NULL, out, HEXCUDA_HMX_OUT_I32, n, n, K, 0);
}
