/* candidate_kernel for i8_matmul_bias_relu_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_matmul_bias_relu_hmx.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, int32_t *out, int n) {
    hexcuda_host_gemm_hmx_ex(A, B, 0, bias, NULL, HEXCUDA_HMX_RES_NONE, NULL, out, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_RELU, 0, n, n, n, 0);
}
