/* candidate_kernel for i8_gemm_bias_relu_requant_hmx on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/i8_gemm_bias_relu_requant_hmx.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias,
                      uint8_t *out, int n) {
    hexcuda_host_gemm_hmx(A, B, 0, bias, out, HEXCUDA_HMX_OUT_U8_BIAS_RELU, n, n, n, 0);
}
