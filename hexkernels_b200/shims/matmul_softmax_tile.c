/* candidate_kernel for matmul_softmax_tile on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/matmul_softmax_tile.h"
void candidate_kernel(const int8_t *Q, const int8_t *K, uint8_t *out, const uint8_t *exp_lut, int32_t inv_sqrt_d, int shift) {
    hexcuda_host_gemm_softmax_u8(Q, K, 1, exp_lut, out, 16, 16, 32, 1, inv_sqrt_d, shift);
}
