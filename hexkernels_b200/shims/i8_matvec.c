/* candidate_kernel for i8_matvec on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_matvec.h"
void candidate_kernel(const int8_t *A, const int8_t *x, int32_t *y, int M, int K) {
    hexcuda_host_gemm_i8_acc(x, 1, A, 1, NULL, NULL, HEXCUDA_HMX_RES_NONE, NULL, y, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, 1, M, K);
}
