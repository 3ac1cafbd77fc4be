/* candidate_kernel for gelu_ffn_residual on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/gelu_ffn_residual.h"
void candidate_kernel(const int8_t *x, const int8_t *W1, const int32_t *b1, const int8_t *gelu_lut, const int8_t *W2, const int32_t *b2, const int8_t *x_res, const int8_t *gamma, const int8_t *beta, const uint8_t *inv_lut, int8_t *out, int M, int K, int V, int D) {
    hexcuda_host_gelu_ffn_residual_i8(x, W1, b1, gelu_lut, W2, b2, x_res, gamma, beta, inv_lut, out, M, K, V, D);
}
