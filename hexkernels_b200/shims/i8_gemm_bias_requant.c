/* candidate_kernel for i8_gemm_bias_requant on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/i8_gemm_bias_requant.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int8_t *out,
                      int M, int N, int K, int32_t mult, int shift, int8_t zp) {
    hexcuda_host_gemm_i8_bias_requant(A, B, bias, out, M, N, K, mult, shift, zp);
}
