/* candidate_kernel for i16_gemm on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i16_gemm.h"
void candidate_kernel(const int16_t *A, const int16_t *B, int32_t *C, int M, int N, int K) {
    hexcuda_host_gemm_i16(A, B, C, M, N, K);
}
