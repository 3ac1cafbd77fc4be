/* candidate_kernel for i8_matmul_add_requant_hmx on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_matmul_add_requant_hmx.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int8_t *residual, int8_t *out, int n) {
    hexcuda_host_gemm_hmx_ex(A, B, 0, NULL, residual, HEXCUDA_HMX_RES_I8, NULL, out, HEXCUDA_HMX_STORE_I8_SAT, HEXCUDA_HMX_ACT_NONE, 0, n, n, n, 0);
}
