/* candidate_kernel for i8_batch_matmul backed by the oracle. */
#include <stddef.h>
#include "kernel_api.h"
#include "hexoracle.h"
void candidate_kernel(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K) {
    for (int b = 0; b < 4; b++)
        oracle_gemm_i8_acc_rows(A + (size_t)b * M * K, 1, B + (size_t)b * K * N, 0, NULL, NULL, 0, NULL, C + (size_t)b * M * N,
                                ORACLE_HMX_STORE_I32, ORACLE_HMX_ACT_NONE, M, N, K, 0, M);
}
