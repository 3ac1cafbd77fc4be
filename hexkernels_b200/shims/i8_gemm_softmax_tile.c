/* candidate_kernel for i8_gemm_softmax_tile on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_gemm_softmax_tile.h"
void candidate_kernel(const int8_t *A, const int8_t *B, uint8_t *out, const uint8_t *exp_lut) {
    hexcuda_host_gemm_softmax_u8(A, B, 0, exp_lut, out, 16, 16, 16, 0, 1, 0);
}
