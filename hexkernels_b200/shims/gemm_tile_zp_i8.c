/* candidate_kernel for gemm_tile_zp_i8 on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/gemm_tile_zp_i8.h"
void candidate_kernel(const int8_t *A, const int8_t *B, int8_t *out, int M, int N, int K,
                      int32_t zpA, int32_t scale_mult, int scale_shift) {
    hexcuda_host_gemm_i8_zp(A, B, out, M, N, K, zpA, scale_mult, scale_shift);
}
