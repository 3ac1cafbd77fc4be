/* candidate_kernel for i8_gemm_tiled_bias_relu_requant on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_gemm_tiled_bias_relu_requant.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, uint8_t *out, int M, int N, int K) {
    hexcuda_host_gemm_hmx_ex(A, B, 0, bias, NULL, HEXCUDA_HMX_RES_NONE, NULL, out, HEXCUDA_HMX_STORE_U8_SAT, HEXCUDA_HMX_ACT_RELU, 0, M, N, K, 0);
}
