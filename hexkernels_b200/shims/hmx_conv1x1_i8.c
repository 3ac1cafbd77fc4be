/* candidate_kernel for hmx_conv1x1_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hmx_conv1x1_i8.h"
void candidate_kernel(const uint8_t *In, const int8_t *W, const int32_t *bias, int32_t *out, int n) {
    hexcuda_host_gemm_hmx_ex(In, W, 1, bias, NULL, HEXCUDA_HMX_RES_NONE, NULL, out, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, 0, n, n, n, 0);
}
