/* candidate_kernel for i8_matmul_bias_gelu_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_matmul_bias_gelu_hmx.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, const int8_t *gelu_lut, int8_t *out, int n) {
    hexcuda_host_gemm_hmx_ex(A, B, 0, bias, NULL, HEXCUDA_HMX_RES_NONE, gelu_lut, out, HEXCUDA_HMX_STORE_LUT_I8, HEXCUDA_HMX_ACT_NONE, 0, n, n, n, 0);
}
