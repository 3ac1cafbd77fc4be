/* candidate_kernel for vtcm_stage_matmul_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/vtcm_stage_matmul_i8.h"
void candidate_kernel(const int8_t *A, const int8_t *X, int32_t *C, int M, int K, int N) {
    hexcuda_host_gemm_i8_acc(A, 1, X, 0, NULL, NULL, HEXCUDA_HMX_RES_NONE, NULL, C, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, M, N, K);
}
