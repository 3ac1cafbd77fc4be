/* candidate_kernel for gemm_bias_relu_requant on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/gemm_bias_relu_requant.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int8_t *out, int M, int N, int K, int32_t mult, int shift, int8_t zp) {
    hexcuda_host_gemm_i8_rq_ex(A, B, 0, bias, NULL, out, M, N, K, mult, shift, zp, 1);
}
