/* candidate_kernel for i8_ffn_block on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_ffn_block.h"
void candidate_kernel(const uint8_t *X, const int8_t *W1, const int32_t *b1, const int8_t *W2, const int32_t *b2, int8_t *out, int S, int D, int Dff) {
    hexcuda_host_ffn_hmx_i8(X, W1, b1, W2, b2, out, S, D, Dff, 8, 3);
}
