/* candidate_kernel for i8_ffn_swiglu_block on the B200 (libhexcuda). */
#include <stddef.h>
#include "hexcuda.h"
#include "kernel_api/i8_ffn_swiglu_block.h"
void candidate_kernel(const uint8_t *X, const int8_t *Wg, const int8_t *Wu, const int8_t *Wd, const int32_t *bd, const uint8_t *silu_lut, int8_t *out, int S, int D, int Dff) {
    hexcuda_host_ffn_swiglu_hmx_i8(X, Wg, Wu, Wd, bd, silu_lut, out, S, D, Dff, 2, 2, 10, 8, 3);
}
