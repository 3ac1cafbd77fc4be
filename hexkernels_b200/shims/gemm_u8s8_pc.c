/* candidate_kernel for the u8 x s8 per-channel GEMM on the B200 (libhexcuda). */
#include "hexcuda.h"
#include "kernel_api/gemm_u8s8_pc.h"
void candidate_kernel(const uint8_t *A, const int8_t *B, const int32_t *bias, uint8_t *out,
                      int M, int N, int K, int32_t zpA, const int32_t *mult, const int *shift,
                      uint8_t zp_out) {
    hexcuda_host_gemm_u8s8_pc(A, B, bias, out, M, N, K, zpA, mult, shift, zp_out);
}
