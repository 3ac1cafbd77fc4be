/* candidate_kernel for av_tile_i8 on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/av_tile_i8.h"
void candidate_kernel(const int8_t *A, const int8_t *V, int32_t *O, int M, int N, int D) {
    hexcuda_host_gemm_i8_acc(A, 1, V, 1, NULL, NULL, HEXCUDA_HMX_RES_NONE, NULL, O, HEXCUDA_HMX_STORE_I32, HEXCUDA_HMX_ACT_NONE, M, D, N);
}
