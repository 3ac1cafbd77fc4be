/* candidate_kernel for i8_batch_matmul_bias on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_batch_matmul_bias.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int32_t *C, int M, int N, int K) {
    for (int b = 0; b < 4; b++)
        if (hexcuda_host_gemm_i8_acc(A + (size_t)b * M * K, 1, B + (size_t)b * K * N, 0, bias + (size_t)b * N, NULL,
                                     HEXCUDA_HMX_RES_NONE, NULL, C + (size_t)b * M * N, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, M, N, K) != HEXCUDA_OK)
            return;
}
