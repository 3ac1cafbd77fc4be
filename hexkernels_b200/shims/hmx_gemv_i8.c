/* candidate_kernel for hmx_gemv_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/hmx_gemv_i8.h"
void candidate_kernel(const uint8_t *A, const int8_t *x, int32_t *out, int n) {
    hexcuda_host_gemm_hmx_ex(A, x, 0, NULL, NULL, HEXCUDA_HMX_RES_NONE, NULL, out, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, 0, n, 1, n, 0);
}
