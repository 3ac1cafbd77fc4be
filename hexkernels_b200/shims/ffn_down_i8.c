/* candidate_kernel for ffn_down_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/ffn_down_i8.h"
void candidate_kernel(const int8_t *A, const int8_t *B, const int32_t *bias, int8_t *out, int M, int N, int K, int32_t scale_mult, int scale_shift) {
    hexcuda_host_gemm_i8_rq_ex(A, B, 1, bias, NULL, out, M, N, K, scale_mult, scale_shift, 0, 0);
}
