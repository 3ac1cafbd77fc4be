/* candidate_kernel for i8_linear_proj_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_linear_proj_hmx.h"
void candidate_kernel(const uint8_t *X, const int8_t *W, const int32_t *bias, int8_t *out, int n) {
    hexcuda_host_gemm_hmx_ex(X, W, 1, bias, NULL, HEXCUDA_HMX_RES_NONE, NULL, out, HEXCUDA_HMX_STORE_I8_SAT, HEXCUDA_HMX_ACT_NONE, 0, n, n, n, 0);
}
