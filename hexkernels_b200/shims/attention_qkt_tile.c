/* candidate_kernel for attention_qkt_tile on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/attention_qkt_tile.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, int8_t *S, int M, int N, int D, int32_t scale_mult, int scale_shift) {
    hexcuda_host_gemm_i8_rq_ex(Q, K, 1, NULL, NULL, S, M, N, D, scale_mult, scale_shift, 0, 0);
}
