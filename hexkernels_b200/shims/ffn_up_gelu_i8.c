/* candidate_kernel for ffn_up_gelu_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/ffn_up_gelu_i8.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, const int8_t *gelu_lut, int8_t *out, int M, int N, int K) {
    hexcuda_host_gemm_i8_acc(A, 1, B, 1, bias, NULL, HEXCUDA_HMX_RES_NONE, gelu_lut, out, HEXCUDA_HMX_STORE_LUT_I8, HEXCUDA_HMX_ACT_NONE, M, N, K);
}
