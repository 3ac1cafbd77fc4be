/* candidate_kernel for qkt_tile_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/qkt_tile_i8.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, int8_t *S, int M, int N, int D, int32_t scale_mult, int scale_shift) {
    hexcuda_host_gemm_i8_rq_ex(Q, K, 0, NULL, NULL, S, M, N, D, scale_mult, scale_shift, 0, 0);
}
